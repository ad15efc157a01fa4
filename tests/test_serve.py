"""Serving surface: OpenAI-compatible HTTP server, vLLM plugin entry point, custom ops."""
import torch

from vllm_xtu_moe_b200.engine import LLM
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.models.config import get_preset


def test_completions_endpoint_cpu():
    from fastapi.testclient import TestClient
    from vllm_xtu_moe_b200.serve import EngineThread, build_app
    llm = LLM(get_preset("tiny-mixtral"), device="cpu",
              runner_config=RunnerConfig(block_size=16, max_seqs=4, max_model_len=256, max_batched_tokens=64,
                                         use_cuda_graph=False))
    eng = EngineThread(llm)
    try:
        c = TestClient(build_app(eng, "tiny-mixtral"))
        assert c.get("/health").json() == {"status": "ok"}
        r = c.post("/v1/completions", json={"prompt": list(range(1, 20)), "max_tokens": 6}).json()
        assert len(r["choices"][0]["token_ids"]) == 6 and r["usage"]["prompt_tokens"] == 19
        r2 = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 3}).json()
        assert r2["usage"]["prompt_tokens"] == 5
        m = c.get("/metrics").text
        assert "xtu_requests_total 2" in m
        # greedy and deterministic: the same prompt gives the same tokens
        r3 = c.post("/v1/completions", json={"prompt": list(range(1, 20)), "max_tokens": 6}).json()
        assert r3["choices"][0]["token_ids"] == r["choices"][0]["token_ids"]
    finally:
        eng.stop()


def test_chat_sampling_and_streaming_cpu():
    import json
    from fastapi.testclient import TestClient
    from vllm_xtu_moe_b200.serve import EngineThread, build_app
    llm = LLM(get_preset("tiny-mixtral"), device="cpu",
              runner_config=RunnerConfig(block_size=16, max_seqs=4, max_model_len=512, max_batched_tokens=64,
                                         use_cuda_graph=False))
    eng = EngineThread(llm)
    try:
        c = TestClient(build_app(eng, "tiny-mixtral"))
        msgs = [{"role": "user", "content": "hi"}]
        r = c.post("/v1/chat/completions", json={"messages": msgs, "max_tokens": 5}).json()
        ch = r["choices"][0]
        assert ch["message"]["role"] == "assistant" and len(ch["token_ids"]) == 5
        assert r["usage"]["completion_tokens"] == 5
        # seeded sampling reproduces; a different seed differs
        body = {"prompt": list(range(1, 20)), "max_tokens": 8, "temperature": 1.5}
        s1 = c.post("/v1/completions", json={**body, "seed": 11}).json()["choices"][0]["token_ids"]
        s2 = c.post("/v1/completions", json={**body, "seed": 11}).json()["choices"][0]["token_ids"]
        s3 = c.post("/v1/completions", json={**body, "seed": 12}).json()["choices"][0]["token_ids"]
        assert s1 == s2 and s1 != s3
        assert c.post("/v1/completions", json={**body, "top_p": 0.0}).status_code == 400
        # n choices: seeds seed, seed + 1 -> the first equals the single seeded call
        multi = c.post("/v1/completions", json={**body, "seed": 11, "n": 2}).json()
        assert [ch["index"] for ch in multi["choices"]] == [0, 1]
        assert multi["choices"][0]["token_ids"] == s1 and multi["choices"][1]["token_ids"] == s3
        lp = c.post("/v1/completions", json={"prompt": list(range(1, 20)), "max_tokens": 4,
                                             "logprobs": 2}).json()["choices"][0]["logprobs"]
        assert len(lp["token_logprobs"]) == 4 and all(len(t) == 2 for t in lp["top_logprobs"])
        # a stop token ends the completion early
        full = c.post("/v1/completions", json={"prompt": list(range(1, 20)), "max_tokens": 8}).json()
        toks = full["choices"][0]["token_ids"]
        cut = c.post("/v1/completions", json={"prompt": list(range(1, 20)), "max_tokens": 8,
                                              "stop_token_ids": [toks[2]]}).json()["choices"][0]
        assert cut["token_ids"] == toks[:toks.index(toks[2]) + 1] and cut["finish_reason"] == "stop"
        # streaming: the events carry the same tokens as the blocking call
        want = c.post("/v1/completions", json={"prompt": list(range(5, 25)), "max_tokens": 7}).json()
        got, done = [], False
        with c.stream("POST", "/v1/completions",
                      json={"prompt": list(range(5, 25)), "max_tokens": 7, "stream": True}) as resp:
            for line in resp.iter_lines():
                if not line.startswith("data: "):
                    continue
                if line == "data: [DONE]":
                    done = True
                    break
                got += json.loads(line[6:])["choices"][0]["token_ids"]
        assert done and got == want["choices"][0]["token_ids"]
        with c.stream("POST", "/v1/chat/completions", json={"messages": msgs, "max_tokens": 4, "stream": True}) as resp:
            events = [l for l in resp.iter_lines() if l.startswith("data: ")]
        assert events[-1] == "data: [DONE]" and "delta" in json.loads(events[0][6:])["choices"][0]
    finally:
        eng.stop()


def test_plugin_registers_custom_ops():
    import vllm_xtu_moe_b200 as pkg
    cfg = pkg.register()
    assert cfg is pkg.register()
    x = torch.randn(3, 64).to(torch.bfloat16)
    w = torch.ones(64).to(torch.bfloat16)
    y = torch.ops.xtu.rmsnorm(x, w, 1e-6)
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    assert (y.float() - ref).abs().max().item() < 2e-2
    assert torch.ops.xtu.argmax(torch.tensor([[0.0, 3.0, 1.0]])).tolist() == [1]
