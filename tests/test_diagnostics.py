"""In-service diagnostics: XIAOTU_DEATH_DEBUG (signal stack dumps + heartbeat) and
XIAOTU_MOE_SELFCHECK (a layer's routed output against its own dequantized weights)."""
import os
import signal
import subprocess
import sys
import textwrap

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_death_debug_logs_signal_stack_and_heartbeat(tmp_path):
    log = tmp_path / "death.log"
    code = textwrap.dedent("""
        import os, sys, time
        sys.path.insert(0, %r)
        import vllm_xtu_moe_b200
        from vllm_xtu_moe_b200.utils import diagnostics as D
        D.set_heartbeat_stats(lambda: {"steps": 7})
        print("ready", flush=True)
        def spin_here():
            time.sleep(30)
        spin_here()
    """ % ROOT)
    env = dict(os.environ, XIAOTU_DEATH_DEBUG="1", XIAOTU_DEATH_LOG=str(log), XIAOTU_DEATH_BEAT_S="0.2")
    p = subprocess.Popen([sys.executable, "-c", code], stdout=subprocess.PIPE, env=env, text=True)
    try:
        assert p.stdout.readline().strip() == "ready"
        import time
        time.sleep(1.0)
        p.send_signal(signal.SIGTERM)
        p.wait(timeout=20)
    finally:
        if p.poll() is None:
            p.kill()
    assert p.returncode == -signal.SIGTERM            # still dies of the signal, after the dump
    text = log.read_text()
    assert "diagnostics on" in text
    assert "alive +" in text and "steps=7" in text
    assert "received signal %d" % signal.SIGTERM in text
    assert "spin_here" in text                         # the main thread's stack at death


def test_death_debug_is_off_by_default():
    from vllm_xtu_moe_b200.utils.diagnostics import install_death_debug
    assert install_death_debug({}) is None


@pytest.mark.parametrize("corrupt", [False, True])
def test_moe_selfcheck_passes_and_catches_a_wrong_weight(corrupt, monkeypatch, capsys):
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.config import get_preset
    from vllm_xtu_moe_b200.models.layers import MoEBlock
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.utils import diagnostics as D
    monkeypatch.setenv("XIAOTU_MOE_SELFCHECK", "1")
    D.SELFCHECK_RESULTS.clear()
    m = build_model(get_preset("tiny-mixtral"), device="cpu", seed=3)
    blocks = [l.mlp for l in m.layers if isinstance(l.mlp, MoEBlock)]
    assert all(b.selfcheck_pending for b in blocks)
    if corrupt:
        # the oracle reads other weights than the executor does: a loading / mapping fault
        b = blocks[0]
        good = b.experts
        bad = type(good)(good.fmt, good.w13 * 1.5, good.w2, good.s13, good.s2, good.interleaved)
        import vllm_xtu_moe_b200.utils.diagnostics as DD
        orig = DD.moe_selfcheck

        def swapped(block, x, ids, w, routed, tol=0.05):
            if block is b:
                block.experts = bad
                try:
                    return orig(block, x, ids, w, routed, tol)
                finally:
                    block.experts = good
            return orig(block, x, ids, w, routed, tol)
        monkeypatch.setattr(DD, "moe_selfcheck", swapped)
    llm = LLM(m, device="cpu", runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=128,
                                                          max_batched_tokens=64, use_cuda_graph=False))
    llm.generate([list(range(1, 20))], SamplingParams(max_tokens=3))
    res = D.SELFCHECK_RESULTS
    assert set(res) == {b.layer_idx for b in blocks}
    if corrupt:
        assert res[blocks[0].layer_idx]["ok"] is False
        assert all(res[b.layer_idx]["ok"] for b in blocks[1:])
    else:
        assert all(r["ok"] for r in res.values()), res
    assert "[xtu-selfcheck]" in capsys.readouterr().err
    D.SELFCHECK_RESULTS.clear()
