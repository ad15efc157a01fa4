"""In-service diagnostics: death debugging and the MoE self-check.

``XIAOTU_DEATH_DEBUG=1`` (the reference's switch, vllm_xiaotu_moe/__init__.py:77-153):
registers faulthandler stack dumps for SIGTERM, SIGINT, SIGHUP, SIGUSR1 and SIGUSR2 (the
signals whose default action ends a process without a traceback), plus a Python handler
for SIGTERM that logs which signal arrived and when, into a file of its own
(``XIAOTU_DEATH_LOG``, default ``/tmp/xtu_sig_<pid>.log``) because a server's stderr may be
redirected or buffered.  A heartbeat thread (``XIAOTU_DEATH_BEAT``, default on, period
``XIAOTU_DEATH_BEAT_S`` seconds) logs that the process is alive, its thread count and the
engine counters a caller registered with :func:`set_heartbeat_stats`.

``XIAOTU_MOE_SELFCHECK=1`` (the reference's switch, vllm_xiaotu_moe/hybrid_model.py:
1612-1750): the first real decode-sized call (at most 64 tokens, non-zero input, not
under CUDA-graph capture) of every MoE layer recomputes its routed-expert output from the
layer's own parameters, dequantized to fp32 by the format's reference decoder, and compares
it with what the layer's executor returned (GPU kernels, pool, ring or CPU engine).  The
verdict is printed once per layer and kept in :data:`SELFCHECK_RESULTS`; a failure means
the weights or activations fed to the executor are not what the model holds (a loading or
mapping fault), not a routing one.
"""
from __future__ import annotations

import faulthandler
import os
import signal
import sys
import threading
import time

import torch

SELFCHECK_RESULTS: dict[int, dict] = {}
_STATS_FN = [None]
_INSTALLED = [False]


def set_heartbeat_stats(fn) -> None:
    """Register a callable returning a short dict of counters for the heartbeat line."""
    _STATS_FN[0] = fn


def install_death_debug(env: dict | None = None) -> str | None:
    """Install the handlers when XIAOTU_DEATH_DEBUG=1; returns the log path (None if off).
    Idempotent within a process."""
    env = os.environ if env is None else env
    if env.get("XIAOTU_DEATH_DEBUG") != "1" or _INSTALLED[0]:
        return None
    _INSTALLED[0] = True
    pid = os.getpid()
    path = env.get("XIAOTU_DEATH_LOG") or f"/tmp/xtu_sig_{pid}.log"
    try:
        fp = open(path, "a", buffering=1)
    except OSError:
        fp, path = sys.stderr, "<stderr>"

    def log(msg: str) -> None:
        print(f"[xtu-death pid={pid} {time.strftime('%H:%M:%S')}] {msg}", file=fp, flush=True)

    faulthandler.enable(file=fp, all_threads=True)
    log("diagnostics on")
    for name in ("SIGTERM", "SIGINT", "SIGHUP", "SIGUSR1", "SIGUSR2"):
        s = getattr(signal, name, None)
        if s is None:
            continue
        try:
            faulthandler.register(s, file=fp, all_threads=True, chain=False)
        except (RuntimeError, ValueError, OSError) as e:
            log(f"faulthandler.register({name}) failed: {e}")

    def on_term(signum, frame):          # the dump does not say which signal came: log it first
        log(f"received signal {signum}")
        faulthandler.dump_traceback(file=fp, all_threads=True)
        fp.flush()
        signal.signal(signal.SIGTERM, signal.SIG_DFL)
        os.kill(os.getpid(), signal.SIGTERM)

    if threading.current_thread() is threading.main_thread():
        try:
            signal.signal(signal.SIGTERM, on_term)
        except (ValueError, OSError) as e:
            log(f"SIGTERM handler not installed: {e}")
    if env.get("XIAOTU_DEATH_BEAT", "1") == "1":
        period = float(env.get("XIAOTU_DEATH_BEAT_S", "10"))
        t0 = time.time()

        def beat():
            while True:
                time.sleep(period)
                extra = ""
                fn = _STATS_FN[0]
                if fn is not None:
                    try:
                        extra = " " + " ".join(f"{k}={v}" for k, v in fn().items())
                    except Exception as e:  # noqa: BLE001 - never let the heartbeat die
                        extra = f" stats-error={type(e).__name__}"
                log(f"alive +{time.time() - t0:.0f}s threads={threading.active_count()}{extra}")

        threading.Thread(target=beat, name="xtu-heartbeat", daemon=True).start()
    return path


def selfcheck_enabled() -> bool:
    return os.environ.get("XIAOTU_MOE_SELFCHECK", "0") == "1"


def moe_selfcheck(block, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, routed: torch.Tensor,
                  tol: float = 0.05) -> dict | None:
    """Compare one MoE call's routed-expert output with an fp32 recomputation from the
    layer's own parameters.  ``routed`` is the executor's output without the shared expert.
    Runs once per layer; returns the verdict (or None when this call does not qualify)."""
    idx = block.layer_idx
    if idx in SELFCHECK_RESULTS:
        return None
    if x.shape[0] == 0 or x.shape[0] > 64:
        return None
    if x.is_cuda and torch.cuda.is_current_stream_capturing():
        return None
    if float(x.detach().abs().max()) == 0.0:        # a dummy / profile input proves nothing
        return None
    from ..ops.moe import moe_ref
    ex = block.experts if block.experts is not None else getattr(block.executor, "reference_experts",
                                                                  lambda b: None)(block)
    if ex is None:
        SELFCHECK_RESULTS[idx] = {"layer": idx, "ok": None, "why": "no dequantizable expert weights here"}
        return SELFCHECK_RESULTS[idx]
    c = block.cfg
    ref = moe_ref(x.float(), ids, w, ex, lo=block.expert_lo, act_limit=c.swiglu_limit).to(routed.device)
    got = routed.float()
    err = float((got - ref).norm() / ref.norm().clamp_min(1e-12))
    res = {"layer": idx, "ok": err <= tol, "rel_err": err, "tokens": int(x.shape[0])}
    SELFCHECK_RESULTS[idx] = res
    print(f"[xtu-selfcheck] layer {idx:02d} tokens={res['tokens']} rel_err={err:.3e} "
          f"{'PASS' if res['ok'] else 'FAIL'}", file=sys.stderr, flush=True)
    return res
