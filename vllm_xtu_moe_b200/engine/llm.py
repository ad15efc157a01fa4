"""Public offline-serving API.

    llm = LLM("glm-4.5-air", device="cuda:0")            # preset name, ModelConfig, or HF dir
    outs = llm.generate([[1, 2, 3], [4, 5]], SamplingParams(max_tokens=32))

``generate`` runs the continuous-batching loop (scheduler -> runner) until every
request finishes and returns the generated token ids with timing (TTFT, decode
window) per request.  Inputs are host token lists; each step copies its
metadata host->device and reads the sampled ids device->host.
"""
from __future__ import annotations

import os
import sys
import time
from dataclasses import dataclass

import torch

from ..config import EngineConfig, get_engine_config
from ..models.config import ModelConfig, get_preset
from ..models.model import MoETransformer, build_model
from .block_manager import BlockManager
from .runner import ModelRunner, RunnerConfig
from .scheduler import Scheduler
from .sequence import Request, SamplingParams, Status


_DEBUG_STEPS = os.environ.get("XTU_DEBUG_STEPS", "0") == "1"


@dataclass
class RequestOutput:
    rid: int
    prompt_len: int
    token_ids: list[int]
    ttft_s: float
    e2e_s: float
    accepted: int = 0
    proposed: int = 0
    logprobs: list | None = None      # per token (log-probability, top alternatives) when asked


class LLM:
    def __init__(self, model: str | ModelConfig | MoETransformer, *, device: str = "cuda", seed: int = 0,
                 runner_config: RunnerConfig | None = None, engine_config: EngineConfig | None = None,
                 tiering=None, num_layers: int | None = None):
        self.econf = engine_config or get_engine_config()
        if isinstance(model, MoETransformer):
            self.model = model
        else:
            ckpt = isinstance(model, str) and os.path.isdir(model)
            if ckpt:
                from ..models.config import from_hf_config
                cfg = from_hf_config(model)
            else:
                cfg = get_preset(model) if isinstance(model, str) else model
            if tiering is None and self.econf.experts_load_device == "cpu":
                # hybrid mode (VLLM_EXPERTS_LOAD_DEVICE=cpu): routed experts on the host tier
                from ..tiering.executor import TieredExperts
                tiering = TieredExperts(cfg, device=device, engine_config=self.econf)
            sink = tiering.expert_sink if tiering is not None else None
            if ckpt:      # HF checkpoint directory (config.json + *.safetensors)
                from ..models.loader import load_model
                self.model, src = load_model(model, device=device, expert_sink=sink, cfg=cfg)
                src.close()
            else:
                self.model = build_model(cfg, device=device, seed=seed, expert_sink=sink, num_layers=num_layers)
        if tiering is not None:
            tiering.attach(self.model)
        self.tiering = tiering
        rc = runner_config or RunnerConfig()
        self.runner = ModelRunner(self.model, rc)
        cfg_m = self.model.cfg
        stateless = not (cfg_m.layer_types and "linear" in cfg_m.layer_types) and rc.swa_blocks == 0
        if rc.prefix_caching and not stateless:
            raise ValueError("prefix caching needs a model without linear-attention state or a sliding-window pool")
        self.blocks = BlockManager(rc.num_blocks, rc.block_size, rc.max_seqs, swa_blocks=rc.swa_blocks,
                                   window=cfg_m.sliding_window, prefix_caching=rc.prefix_caching)
        self.scheduler = Scheduler(self.blocks, rc.max_batched_tokens, rc.max_seqs, rc.num_spec)
        self.spec = None
        self.max_spec = rc.num_spec
        if rc.num_spec > 0 and self.model.mtp:
            from .spec_decode import SpecDecoder
            self.spec = SpecDecoder(self.runner, rc.num_spec, self.blocks)
        self.stats = dict(prefill_tokens=0, decode_tokens=0, prefill_time=0.0, decode_time=0.0, steps=0)
        self.tracer = None
        ec = self.econf
        if ec.routing_dump or ec.layer_timing or ec.torch_profile or ec.nvtx:
            from ..utils.trace import Tracer
            self.tracer = Tracer(self.model, ec)
            self.model.attach_tracer(self.tracer)

    # ------------------------------------------------------------------
    def set_speculation(self, k: int) -> None:
        """Change the MTP draft count between requests (0 = plain decoding), up to the
        ``num_spec`` the runner was built with (its block reservations and workspaces are
        sized for that); only while no request is in flight."""
        if self.scheduler.has_work():
            raise RuntimeError("set_speculation while requests are in flight")
        if k < 0 or k > self.max_spec:
            raise ValueError(f"k must lie in [0, {self.max_spec}]")
        if k > 0 and not self.model.mtp:
            raise ValueError("speculative decoding needs a model with an MTP layer")
        if self.spec is not None:
            self.spec.release_graphs()
        self.runner.rc.num_spec = k
        self.scheduler.num_spec = k
        self.spec = None
        if k > 0:
            from .spec_decode import SpecDecoder
            self.spec = SpecDecoder(self.runner, k, self.blocks)

    # ------------------------------------------------------------------
    def check_request(self, prompt: list[int], params: SamplingParams) -> None:
        """Raise ValueError for a request this engine cannot serve (called by add_request;
        the server calls it before queueing, so a bad request gets an HTTP 400 and never
        reaches the engine thread)."""
        if params.logprobs is not None and self.spec is not None:
            raise ValueError("token log-probabilities with speculative decoding are not supported: use num_spec=0")
        if not prompt:
            raise ValueError("empty prompt")
        if params.max_tokens < 1:
            raise ValueError("max_tokens must be at least 1")
        rc = self.runner.rc
        n = len(prompt) + params.max_tokens
        if n > rc.max_model_len:
            raise ValueError(f"prompt ({len(prompt)} tokens) + max_tokens ({params.max_tokens}) = {n} exceeds "
                             f"max_model_len ({rc.max_model_len})")
        vocab = self.model.cfg.vocab_size
        if min(prompt) < 0 or max(prompt) >= vocab:
            raise ValueError(f"token ids must lie in [0, {vocab})")

    def add_request(self, prompt: list[int], params: SamplingParams) -> Request:
        self.check_request(prompt, params)
        r = Request(list(prompt), params)
        r.t_submit = time.perf_counter()
        self.scheduler.add(r)
        return r

    def abort(self, rid: int) -> bool:
        """Stop request `rid` between steps (e.g. its client went away); its blocks and
        recurrent-state slot are freed.  Returns whether the request was still live."""
        return self.scheduler.abort(rid) is not None

    def step(self, plan=None) -> list[Request]:
        """Run one engine step (scheduling it unless a plan is given); returns finished requests."""
        if plan is None:
            plan = self.scheduler.schedule()
        if plan is None:
            return []
        if self.tracer is not None and self.tracer.profiler is not None:
            self.tracer.profiler.before_step()
        try:
            return self._step(plan)
        finally:
            if self.tracer is not None:
                if self.tracer.profiler is not None:
                    self.tracer.profiler.after_step()
                if self.tracer.routing is not None:
                    self.tracer.routing.end_step()

    def _step(self, plan) -> list[Request]:
        t0 = time.perf_counter()
        if plan.is_decode and self.spec is not None:
            done = self.spec.decode_step(plan, self.scheduler)
            self.stats["decode_time"] += time.perf_counter() - t0
            self.stats["steps"] += 1
            if self.tiering is not None:
                self.tiering.step_done()
            return done
        tok, extra = self.runner.execute(plan)
        toks = tok.tolist() if tok is not None else []
        if tok is not None:
            self.runner.d2h_bytes += tok.numel() * tok.element_size()
        now = time.perf_counter()
        if _DEBUG_STEPS:
            print(f"[xtu-step] {'decode' if plan.is_decode else 'prefill'} seqs={len(plan.chunks)} "
                  f"tokens={plan.num_tokens} {1e3 * (now - t0):.1f} ms", file=sys.stderr, flush=True)
        done = []
        if plan.is_decode:
            for ch, t in zip(plan.chunks, toks):
                r = ch.req
                r.num_computed = r.total_len
                r.output.append(int(t))
                self.stats["decode_tokens"] += 1
                if r.finished():
                    r.t_done = now
                    self.scheduler.finish(r)
                    done.append(r)
            self.stats["decode_time"] += now - t0
        else:
            it = iter(toks)
            for ch in plan.chunks:
                r = ch.req
                r.num_computed += ch.length
                self.stats["prefill_tokens"] += ch.length
                if r.num_computed == len(r.prompt):
                    r.output.append(int(next(it)))
                    r.t_first = now
                    r.status = Status.DECODE
                    if self.spec is not None:
                        self.spec.after_prefill(r, extra)
                    if r.finished():
                        r.t_done = now
                        self.scheduler.finish(r)
                        done.append(r)
            if self.spec is not None:
                self.spec.prefill_mtp(plan, extra)
            self.stats["prefill_time"] += now - t0
        self.stats["steps"] += 1
        if self.tiering is not None:
            self.tiering.step_done()
        return done

    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None):
        params = params or SamplingParams()
        ps = params if isinstance(params, list) else [params] * len(prompts)
        reqs = [self.add_request(p, sp) for p, sp in zip(prompts, ps)]
        while self.scheduler.has_work():
            self.step()
        out = []
        for r in reqs:
            out.append(RequestOutput(r.rid, len(r.prompt), list(r.output), r.t_first - r.t_submit,
                                     r.t_done - r.t_submit, r.accepted, r.proposed,
                                     list(r.logprobs) if r.params.logprobs is not None else None))
        return out

    def shutdown(self):
        self.runner.release_graphs()
        if self.spec is not None:
            self.spec.release_graphs()
        if self.tracer is not None:
            self.tracer.close()
        if self.tiering is not None:
            self.tiering.shutdown()
