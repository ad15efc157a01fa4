"""Request admission and KV-pool pressure: requests larger than the pool or than
max_model_len are rejected up front, prompts in prefill that together exceed the pool
make progress (the newest goes back to the queue), and the server answers 400 for a
request it cannot serve instead of failing its engine thread."""
import pytest

from vllm_xtu_moe_b200.engine import LLM, SamplingParams
from vllm_xtu_moe_b200.engine.block_manager import BlockManager
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.engine.scheduler import Scheduler
from vllm_xtu_moe_b200.engine.sequence import Request, Status
from vllm_xtu_moe_b200.models.config import get_preset


def _drive(sched: Scheduler, max_steps: int = 10_000) -> int:
    """Play the engine's role (no model): advance every scheduled chunk, emit one token per
    decode row.  Returns the number of steps taken; fails on a step with nothing to run."""
    steps = 0
    while sched.has_work():
        plan = sched.schedule()
        assert plan is not None, "scheduler has work but schedules nothing (would spin forever)"
        steps += 1
        assert steps < max_steps
        for ch in plan.chunks:
            r = ch.req
            if plan.is_decode:
                r.num_computed = r.total_len
                r.output.append(1)
                if r.finished():
                    sched.finish(r)
            else:
                r.num_computed += ch.length
                if r.num_computed == len(r.prompt):
                    r.output.append(1)
                    r.status = Status.DECODE
                    if r.finished():
                        sched.finish(r)
    return steps


def test_prompts_in_prefill_that_exceed_the_pool_together_make_progress():
    bm = BlockManager(num_blocks=20, block_size=16, max_seqs=4)     # 320 tokens of KV
    s = Scheduler(bm, max_batched_tokens=64, max_seqs=4)
    a = Request(list(range(250)), SamplingParams(max_tokens=8))
    b = Request(list(range(250)), SamplingParams(max_tokens=8))
    s.add(a)
    s.add(b)
    _drive(s)
    assert len(a.output) == 8 and len(b.output) == 8
    assert bm.num_free == 20


def test_request_larger_than_the_pool_is_rejected():
    bm = BlockManager(num_blocks=4, block_size=16, max_seqs=2)
    s = Scheduler(bm, max_batched_tokens=64, max_seqs=2)
    with pytest.raises(ValueError, match="KV cache"):
        s.add(Request(list(range(60)), SamplingParams(max_tokens=16)))
    s.add(Request(list(range(30)), SamplingParams(max_tokens=10)))
    _drive(s)


def _tiny_llm():
    return LLM(get_preset("tiny-mixtral"), device="cpu",
               runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=64, max_batched_tokens=64,
                                          use_cuda_graph=False))


def test_over_long_request_is_rejected_by_add_request():
    llm = _tiny_llm()
    with pytest.raises(ValueError, match="max_model_len"):
        llm.add_request(list(range(1, 60)), SamplingParams(max_tokens=10))
    with pytest.raises(ValueError, match="token ids"):
        llm.add_request([1, 2, 10 ** 6], SamplingParams(max_tokens=2))
    out = llm.generate([list(range(1, 40))], SamplingParams(max_tokens=4))
    assert len(out[0].token_ids) == 4


def test_server_answers_400_for_an_over_long_request_and_keeps_serving():
    from fastapi.testclient import TestClient
    from vllm_xtu_moe_b200.serve import EngineThread, build_app
    llm = _tiny_llm()
    eng = EngineThread(llm)
    try:
        c = TestClient(build_app(eng, "tiny-mixtral"))
        r = c.post("/v1/completions", json={"prompt": list(range(1, 60)), "max_tokens": 10})
        assert r.status_code == 400 and "max_model_len" in r.json()["detail"]
        r = c.post("/v1/completions", json={"prompt": list(range(1, 60)), "max_tokens": 10, "stream": True})
        assert r.status_code == 400
        ok = c.post("/v1/completions", json={"prompt": list(range(1, 20)), "max_tokens": 3}).json()
        assert len(ok["choices"][0]["token_ids"]) == 3
        assert c.get("/health").json() == {"status": "ok"}
    finally:
        eng.stop()


def test_abort_before_admission_drops_the_request():
    from concurrent.futures import Future
    from vllm_xtu_moe_b200.serve import EngineThread
    llm = _tiny_llm()
    eng = EngineThread(llm)
    try:
        eng._stop.set()            # park the loop so the abort arrives while the request is queued
        eng.thread.join(timeout=10)
        f: Future = eng.submit(list(range(1, 20)), SamplingParams(max_tokens=3))
        eng.abort(f)
        # run one loop iteration by hand: the abort is seen first, then the inbox
        eng._stop.clear()
        while not eng.aborts.empty():
            fut = eng.aborts.get_nowait()
            eng._cancelled.add(fut)
        import threading
        t = threading.Thread(target=eng._loop, daemon=True)
        t.start()
        import time
        t_end = time.time() + 10
        while not f.done() and time.time() < t_end:
            time.sleep(0.01)
        assert f.cancelled()
        assert not llm.scheduler.has_work()
    finally:
        eng.stop()
        eng._stop.set()
