"""OpenAI-compatible HTTP server over the engine (replaces the reference's
``vllm.entrypoints.openai.api_server`` launch, scripts/serve_v41.sh:637-664).

    python -m vllm_xtu_moe_b200.serve --model glm-4.5-air --port 8000 [--num-spec 4]

Endpoints: ``POST /v1/completions`` (prompt = token ids, or text encoded as UTF-8
bytes when no tokenizer is configured), ``GET /v1/models``, ``GET /health`` and
``GET /metrics`` (Prometheus: requests, generated tokens, time to first token, step
latency).  One engine thread owns the GPU: HTTP handlers enqueue requests and wait
on a future; the thread admits new requests between steps (continuous batching).
"""

import argparse
import asyncio
import queue
import threading
import time
from concurrent.futures import Future

from .engine import LLM, SamplingParams
from .engine.runner import RunnerConfig


class EngineThread:
    """Runs ``LLM.step`` in a loop on one thread; ``submit`` is thread-safe."""

    def __init__(self, llm: LLM):
        self.llm = llm
        self.inbox: queue.Queue = queue.Queue()
        self.pending: dict[int, tuple[Future, float]] = {}
        self.metrics = {"requests": 0, "tokens": 0, "steps": 0}
        self._stop = threading.Event()
        self.error: BaseException | None = None
        self.thread = threading.Thread(target=self._loop, name="xtu-engine", daemon=True)
        self.thread.start()

    def submit(self, prompt: list[int], params: SamplingParams) -> Future:
        f: Future = Future()
        self.inbox.put((prompt, params, f))
        return f

    def _loop(self):
        try:
            while not self._stop.is_set():
                admitted = False
                while True:
                    try:
                        prompt, params, f = self.inbox.get_nowait()
                    except queue.Empty:
                        break
                    r = self.llm.add_request(prompt, params)
                    self.pending[r.rid] = (f, time.perf_counter())
                    admitted = True
                if not self.llm.scheduler.has_work():
                    if not admitted:
                        time.sleep(0.001)
                    continue
                done = self.llm.step()
                self.metrics["steps"] += 1
                for r in done:
                    f, _ = self.pending.pop(r.rid)
                    self.metrics["requests"] += 1
                    self.metrics["tokens"] += len(r.output)
                    f.set_result(r)
        except BaseException as e:      # surface engine failures to every waiter
            self.error = e
            for f, _ in self.pending.values():
                f.set_exception(e)

    def stop(self):
        self._stop.set()
        self.thread.join(timeout=10)


def _encode(prompt) -> list[int]:
    if isinstance(prompt, list):
        return [int(t) for t in prompt]
    return list(str(prompt).encode("utf-8"))


def build_app(engine: EngineThread, model_name: str):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse
    from pydantic import BaseModel

    class CompletionRequest(BaseModel):
        model: str | None = None
        prompt: list[int] | str
        max_tokens: int = 16
        temperature: float = 0.0
        ignore_eos: bool = True

    app = FastAPI(title="vllm_xtu_moe_b200")

    @app.get("/health")
    def health():
        if engine.error is not None:
            raise HTTPException(500, repr(engine.error))
        return {"status": "ok"}

    @app.get("/v1/models")
    def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model"}]}

    @app.get("/metrics", response_class=PlainTextResponse)
    def metrics():
        m = engine.metrics
        st = engine.llm.stats
        lines = [f"xtu_requests_total {m['requests']}", f"xtu_generated_tokens_total {m['tokens']}",
                 f"xtu_engine_steps_total {m['steps']}", f"xtu_prefill_tokens_total {st['prefill_tokens']}",
                 f"xtu_decode_tokens_total {st['decode_tokens']}",
                 f"xtu_prefill_seconds_total {st['prefill_time']:.6f}",
                 f"xtu_decode_seconds_total {st['decode_time']:.6f}"]
        return "\n".join(lines) + "\n"

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        if req.temperature != 0.0:
            raise HTTPException(400, "only greedy decoding (temperature 0) is served")
        ids = _encode(req.prompt)
        fut = engine.submit(ids, SamplingParams(max_tokens=req.max_tokens, ignore_eos=req.ignore_eos))
        r = await asyncio.wrap_future(fut)
        return {"id": f"cmpl-{r.rid}", "object": "text_completion", "model": model_name,
                "choices": [{"index": 0, "token_ids": list(r.output), "finish_reason": "length"}],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(r.output),
                          "total_tokens": len(ids) + len(r.output)},
                "timing": {"ttft_s": r.t_first - r.t_submit, "e2e_s": r.t_done - r.t_submit}}

    return app


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="glm-4.5-air")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--max-seqs", type=int, default=8)
    ap.add_argument("--max-model-len", type=int, default=32768)
    ap.add_argument("--max-batched-tokens", type=int, default=16384)
    ap.add_argument("--num-spec", type=int, default=0)
    ap.add_argument("--layers", type=int, default=None)
    a = ap.parse_args(argv)
    import uvicorn
    rc = RunnerConfig(max_seqs=a.max_seqs, max_model_len=a.max_model_len, max_batched_tokens=a.max_batched_tokens,
                      num_spec=a.num_spec)
    llm = LLM(a.model, device=a.device, runner_config=rc, num_layers=a.layers)
    eng = EngineThread(llm)
    uvicorn.run(build_app(eng, a.model), host=a.host, port=a.port, log_level="warning")
    eng.stop()
    llm.shutdown()


if __name__ == "__main__":
    main()
