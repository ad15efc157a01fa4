"""OpenAI-compatible HTTP server over the engine (replaces the reference's
``vllm.entrypoints.openai.api_server`` launch, scripts/serve_v41.sh:637-664).

    python -m vllm_xtu_moe_b200.serve --model glm-4.5-air --port 8000 [--num-spec 4]
        [--tokenizer /path/to/hf/tokenizer]

Endpoints: ``POST /v1/completions`` (prompt = token ids or text) and
``POST /v1/chat/completions`` (messages), both with greedy or sampled decoding
(temperature, top_p, top_k, seed) and ``"stream": true`` (server-sent events, one event
per engine step that produced tokens, then ``data: [DONE]``); ``GET /v1/models``,
``GET /health`` and ``GET /metrics`` (Prometheus text).  Text goes through a HF tokenizer
from a local directory when one is given, else through UTF-8 bytes (token id = byte).
One engine thread owns the GPU: HTTP handlers enqueue requests and wait on a future (or
a per-request queue when streaming); the thread admits new requests between steps
(continuous batching).
"""

import argparse
import asyncio
import dataclasses
import json
import queue
import threading
import time
from concurrent.futures import Future

from .engine import LLM, SamplingParams
from .engine.runner import RunnerConfig


class EngineThread:
    """Runs ``LLM.step`` in a loop on one thread; ``submit`` is thread-safe.  ``on_tokens``
    (optional) is called on the engine thread after every step that gave the request new
    tokens, with (new token ids, finished)."""

    def __init__(self, llm: LLM):
        self.llm = llm
        self.inbox: queue.Queue = queue.Queue()
        self.pending: dict[int, tuple[Future, float]] = {}
        self.streams: dict[int, list] = {}          # rid -> [callback, tokens already sent, request]
        self.metrics = {"requests": 0, "tokens": 0, "steps": 0, "aborted": 0, "ttft_s": 0.0, "e2e_s": 0.0}
        self.aborts: queue.Queue = queue.Queue()
        self._cancelled: set = set()     # aborted futures whose request was not admitted yet
        self._stop = threading.Event()
        self.error: BaseException | None = None
        self.thread = threading.Thread(target=self._loop, name="xtu-engine", daemon=True)
        self.thread.start()

    def submit(self, prompt: list[int], params: SamplingParams, on_tokens=None) -> Future:
        f: Future = Future()
        self.inbox.put((prompt, params, f, on_tokens))
        return f

    def abort(self, fut: Future) -> None:
        """Cancel the request behind `fut` at the next step boundary (thread-safe)."""
        self.aborts.put(fut)

    def _push(self, r, done: bool) -> None:
        st = self.streams.get(r.rid)
        if st is None:
            return
        cb, sent, _ = st
        new = list(r.output[sent:])
        if new or done:
            st[1] = len(r.output)
            cb(new, done)
        if done:
            del self.streams[r.rid]

    def _loop(self):
        try:
            while not self._stop.is_set():
                admitted = False
                while True:
                    try:
                        prompt, params, f, cb = self.inbox.get_nowait()
                    except queue.Empty:
                        break
                    if f in self._cancelled:      # its client went away before admission
                        self._cancelled.discard(f)
                        self.metrics["aborted"] += 1
                        f.cancel()
                        if cb is not None:
                            cb([], True)
                        continue
                    try:
                        r = self.llm.add_request(prompt, params)
                    except ValueError as e:       # a request this engine cannot serve
                        f.set_exception(e)
                        continue
                    self.pending[r.rid] = (f, time.perf_counter())
                    if cb is not None:
                        self.streams[r.rid] = [cb, 0, r]
                    admitted = True
                while True:              # cancellations (clients that went away)
                    try:
                        fut = self.aborts.get_nowait()
                    except queue.Empty:
                        break
                    found = False
                    for rid, (f, _) in list(self.pending.items()):
                        if f is fut:
                            found = True
                            if self.llm.abort(rid):
                                self.pending.pop(rid)
                                self.streams.pop(rid, None)
                                self.metrics["aborted"] += 1
                                f.cancel()
                    if not found and not fut.done():
                        self._cancelled.add(fut)  # still in the inbox: dropped when it is drained
                if not self.llm.scheduler.has_work():
                    if not admitted:
                        time.sleep(0.001)
                    continue
                done = self.llm.step()
                self.metrics["steps"] += 1
                done_ids = {r.rid for r in done}
                for st in list(self.streams.values()):
                    if st[2].rid not in done_ids:
                        self._push(st[2], False)
                for r in done:
                    self._push(r, True)
                    f, _ = self.pending.pop(r.rid)
                    self.metrics["requests"] += 1
                    self.metrics["tokens"] += len(r.output)
                    self.metrics["ttft_s"] += r.t_first - r.t_submit
                    self.metrics["e2e_s"] += r.t_done - r.t_submit
                    f.set_result(r)
        except BaseException as e:      # surface engine failures to every waiter
            self.error = e
            for f, _ in self.pending.values():
                if not f.done():
                    f.set_exception(e)
            for cb, _, _ in self.streams.values():
                cb([], True)

    def stop(self):
        self._stop.set()
        self.thread.join(timeout=10)


class TextCodec:
    """Text <-> token ids: a HF tokenizer loaded from a local directory, or UTF-8 bytes."""

    def __init__(self, tokenizer_path: str | None = None):
        self.tok = None
        if tokenizer_path:
            from transformers import AutoTokenizer
            self.tok = AutoTokenizer.from_pretrained(tokenizer_path, local_files_only=True)

    def encode(self, prompt) -> list[int]:
        if isinstance(prompt, list):
            return [int(t) for t in prompt]
        if self.tok is not None:
            return list(self.tok.encode(str(prompt)))
        return list(str(prompt).encode("utf-8"))

    def decode(self, ids: list[int]) -> str:
        if self.tok is not None:
            return self.tok.decode(ids)
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def chat(self, messages: list[dict]) -> list[int]:
        if self.tok is not None and getattr(self.tok, "chat_template", None):
            return list(self.tok.apply_chat_template(messages, add_generation_prompt=True))
        text = "".join(f"{m.get('role', 'user')}: {m.get('content', '')}\n" for m in messages) + "assistant: "
        return self.encode(text)

    @property
    def eos(self) -> int | None:
        return getattr(self.tok, "eos_token_id", None) if self.tok is not None else None


def _encode(prompt) -> list[int]:
    return TextCodec().encode(prompt)


def build_app(engine: EngineThread, model_name: str, codec: TextCodec | None = None):
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import PlainTextResponse, StreamingResponse
    from pydantic import BaseModel

    codec = codec or TextCodec()

    class Sampling(BaseModel):
        model: str | None = None
        max_tokens: int = 16
        temperature: float = 0.0
        top_p: float = 1.0
        top_k: int = 0
        seed: int | None = None
        ignore_eos: bool = True
        stop_token_ids: list[int] = []
        stream: bool = False
        n: int = 1                       # choices per request (sampled: seeds seed, seed+1, ...)
        logprobs: int | None = None      # per-token log-probabilities and this many alternatives

    class CompletionRequest(Sampling):
        prompt: list[int] | str

    class ChatRequest(Sampling):
        messages: list[dict]

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
                 f"xtu_requests_aborted_total {m['aborted']}",
                 f"xtu_time_to_first_token_seconds_sum {m['ttft_s']:.6f}",
                 f"xtu_request_latency_seconds_sum {m['e2e_s']:.6f}",
                 f"xtu_engine_steps_total {m['steps']}", f"xtu_prefill_tokens_total {st['prefill_tokens']}",
                 f"xtu_decode_tokens_total {st['decode_tokens']}",
                 f"xtu_prefill_seconds_total {st['prefill_time']:.6f}",
                 f"xtu_decode_seconds_total {st['decode_time']:.6f}"]
        tier = getattr(engine.llm, "tiering", None)
        if tier is not None:
            ts = tier.stats(hit_rate=False)
            lines += [f"xtu_tier_calls_total{{path=\"{k}\"}} {v}" for k, v in ts.items() if k != "swaps"]
            lines.append(f"xtu_pool_swaps_total {ts['swaps']}")
        return "\n".join(lines) + "\n"

    def params_of(req: Sampling) -> SamplingParams:
        if req.temperature < 0 or not (0 < req.top_p <= 1) or req.top_k < 0 or req.max_tokens < 1:
            raise HTTPException(400, "invalid sampling parameters")
        return SamplingParams(max_tokens=req.max_tokens, temperature=req.temperature, top_p=req.top_p,
                              top_k=req.top_k, seed=req.seed, ignore_eos=req.ignore_eos, eos_token_id=codec.eos,
                              stop_token_ids=tuple(req.stop_token_ids),
                              logprobs=None if req.logprobs is None else max(0, min(int(req.logprobs), 20)))

    async def run(ids: list[int], sp: SamplingParams):
        check(ids, sp)
        try:
            return await asyncio.wrap_future(engine.submit(ids, sp))
        except ValueError as e:
            raise HTTPException(400, str(e))

    async def run_n(ids: list[int], sp: SamplingParams, n: int):
        """n choices: n requests (batched by the engine), seeds seed, seed + 1, ..."""
        if n < 1 or n > 64:
            raise HTTPException(400, "n must be in [1, 64]")
        sps = [sp if i == 0 else dataclasses.replace(sp, seed=None if sp.seed is None else sp.seed + i)
               for i in range(n)]
        return await asyncio.gather(*(run(ids, p) for p in sps))

    def check(ids: list[int], sp: SamplingParams) -> None:
        try:
            engine.llm.check_request(ids, sp)
        except ValueError as e:
            raise HTTPException(400, str(e))

    def stream(ids: list[int], sp: SamplingParams, make_chunk):
        check(ids, sp)
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        fut = engine.submit(ids, sp, on_tokens=lambda new, done: loop.call_soon_threadsafe(q.put_nowait, (new, done)))

        async def events():
            finished = False
            try:
                while True:
                    new, done = await q.get()
                    if new:
                        yield "data: " + json.dumps(make_chunk(new)) + "\n\n"
                    if done:
                        finished = True
                        yield "data: [DONE]\n\n"
                        return
            finally:
                if not finished:        # the client went away: stop generating for it
                    engine.abort(fut)
        return StreamingResponse(events(), media_type="text/event-stream")

    def logprobs_of(r):
        if r.params.logprobs is None:
            return None
        return {"tokens": list(r.output), "token_logprobs": [lp for lp, _ in r.logprobs],
                "top_logprobs": [{str(t): v for t, v in alt.items()} for _, alt in r.logprobs]}

    def usage(ids, out):
        return {"prompt_tokens": len(ids), "completion_tokens": len(out), "total_tokens": len(ids) + len(out)}

    @app.post("/v1/completions")
    async def completions(req: CompletionRequest):
        ids = codec.encode(req.prompt)
        sp = params_of(req)
        if req.stream:
            if req.n != 1:
                raise HTTPException(400, "streaming serves one choice (n = 1)")
            return stream(ids, sp, lambda new: {"object": "text_completion", "model": model_name, "choices": [
                {"index": 0, "token_ids": new, "text": codec.decode(new), "finish_reason": None}]})
        rs = await run_n(ids, sp, req.n)
        r = rs[0]
        return {"id": f"cmpl-{r.rid}", "object": "text_completion", "model": model_name,
                "choices": [{"index": i, "token_ids": list(x.output), "text": codec.decode(list(x.output)),
                             "logprobs": logprobs_of(x),
                             "finish_reason": "length" if len(x.output) >= sp.max_tokens else "stop"}
                            for i, x in enumerate(rs)],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": sum(len(x.output) for x in rs),
                          "total_tokens": len(ids) + sum(len(x.output) for x in rs)},
                "timing": {"ttft_s": r.t_first - r.t_submit, "e2e_s": r.t_done - r.t_submit}}

    @app.post("/v1/chat/completions")
    async def chat(req: ChatRequest):
        ids = codec.chat(req.messages)
        sp = params_of(req)
        if req.stream:
            return stream(ids, sp, lambda new: {"object": "chat.completion.chunk", "model": model_name, "choices": [
                {"index": 0, "delta": {"content": codec.decode(new)}, "token_ids": new, "finish_reason": None}]})
        r = await run(ids, sp)
        out = list(r.output)
        return {"id": f"chatcmpl-{r.rid}", "object": "chat.completion", "model": model_name,
                "choices": [{"index": 0, "message": {"role": "assistant", "content": codec.decode(out)},
                             "token_ids": out, "finish_reason": "length" if len(out) >= sp.max_tokens else "stop"}],
                "usage": usage(ids, out)}

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
    ap.add_argument("--tokenizer", default=None, help="local HF tokenizer directory (default: UTF-8 bytes)")
    ap.add_argument("--prefix-caching", action="store_true", help="reuse the KV blocks of cached prompt prefixes")
    a = ap.parse_args(argv)
    import uvicorn
    rc = RunnerConfig(max_seqs=a.max_seqs, max_model_len=a.max_model_len, max_batched_tokens=a.max_batched_tokens,
                      num_spec=a.num_spec, prefix_caching=a.prefix_caching)
    llm = LLM(a.model, device=a.device, runner_config=rc, num_layers=a.layers)
    eng = EngineThread(llm)
    uvicorn.run(build_app(eng, a.model, TextCodec(a.tokenizer)), host=a.host, port=a.port, log_level="warning")
    eng.stop()
    llm.shutdown()


if __name__ == "__main__":
    main()
