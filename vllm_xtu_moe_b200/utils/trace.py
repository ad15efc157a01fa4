"""Observability: routing capture, NVTX ranges, per-layer timing, torch-profiler window.

* Routing dump (``XIAOTU_ROUTING_DUMP=<file>``): every MoE layer adds its step's
  top-k ids into a device counter matrix [layers, E] with ``index_add_`` (static
  shapes, so decode graphs capture it); nothing is read back until ``flush``, which
  writes ``{"experts": E, "counts": {layer: [...]}}`` as JSON.  ``to_xtup`` turns a
  dump into an XTUP hot-expert table (the reference's routing-dump -> pin-table
  tooling: binding.cpp:468-565 ring + scripts/expert_profile.py).
* NVTX (``XIAOTU_NVTX=1``): named ranges around layers and engine steps.
* Layer timing (``XIAOTU_LAYER_TIMING=1``, eager steps only): CUDA events around each
  decoder layer; ``LayerTimer.report`` gives mean milliseconds per layer.
* Torch profiler (``XIAOTU_TORCH_PROFILE=<dir>[:first:count]``): records steps
  [first, first+count) to a Chrome trace, never while a CUDA graph is being captured
  (the reference's hooks, hybrid_model.py:336-417).
"""
from __future__ import annotations

import contextlib
import json
import os
import sys
from pathlib import Path

import torch

from ..config import get_engine_config


class RoutingDump:
    """Device routing counters plus per-window deltas: every ``window`` engine steps
    (``XIAOTU_ROUTING_DUMP_WINDOW``, default 16) ``end_step`` keeps the counts added since
    the last window (a device-side copy, no read-back), so the PIN tooling can evaluate a
    table on windows it was not built from (``tiering.pin_tools``).  Past ``max_windows``
    adjacent windows are merged pairwise, which keeps memory bounded on long runs."""

    def __init__(self, path: str, num_layers: int, num_experts: int, device, window: int | None = None,
                 max_windows: int = 4096):
        self.path = path
        self.E = num_experts
        self.counts = torch.zeros(num_layers, num_experts, dtype=torch.int64, device=device)
        self._ones = {}
        self.window = window if window is not None else max(1, int(os.environ.get("XIAOTU_ROUTING_DUMP_WINDOW",
                                                                                 "16")))
        self.max_windows = max_windows
        self._steps = 0
        self._cut_at = 0
        self._last = torch.zeros_like(self.counts)
        self.windows: list[torch.Tensor] = []

    def end_step(self) -> None:
        self._steps += 1
        if self._steps % self.window:
            return
        self._cut()

    def _cut(self) -> None:
        if self._steps == self._cut_at:        # nothing recorded since the last window
            return
        self._cut_at = self._steps
        self.windows.append(self.counts - self._last)
        self._last = self.counts.clone()
        if len(self.windows) > self.max_windows:
            w = self.windows
            self.windows = [w[i] + w[i + 1] if i + 1 < len(w) else w[i] for i in range(0, len(w), 2)]

    def record(self, layer: int, ids: torch.Tensor) -> None:
        flat = ids.reshape(-1).long()
        key = (flat.numel(), flat.device)
        ones = self._ones.get(key)
        if ones is None:
            ones = torch.ones(flat.numel(), dtype=torch.int64, device=flat.device)
            self._ones[key] = ones
        self.counts[layer].index_add_(0, flat.clamp_(0, self.E - 1), ones)

    def flush(self) -> str:
        self._cut()
        c = self.counts.cpu().tolist()
        wins = []
        for w in self.windows:
            rows = w.cpu().tolist()
            wins.append({str(l): row for l, row in enumerate(rows) if any(row)})
        data = {"experts": self.E, "counts": {str(l): row for l, row in enumerate(c) if any(row)},
                "window_steps": self.window, "windows": [w for w in wins if w]}
        Path(self.path).write_text(json.dumps(data))
        return self.path


def load_dump(path: str) -> tuple[int, dict[int, list[int]]]:
    d = json.loads(Path(path).read_text())
    return d["experts"], {int(k): v for k, v in d["counts"].items()}


def load_windows(path: str) -> list[dict[int, list[int]]]:
    """The dump's per-window count deltas (layer -> per-expert counts), oldest first."""
    d = json.loads(Path(path).read_text())
    return [{int(k): v for k, v in w.items()} for w in d.get("windows", [])]


def to_xtup(dump_path: str, out_path: str, per_layer: int) -> dict:
    """Routing dump -> XTUP table of the per_layer hottest experts; returns coverage stats."""
    from ..tiering.policy import save_pin_table, table_from_counts
    E, counts = load_dump(dump_path)
    table = table_from_counts(counts, per_layer)
    save_pin_table(out_path, table, E)
    cov = {}
    for l, c in counts.items():
        tot = sum(c)
        cov[l] = sum(c[e] for e in table.get(l, [])) / tot if tot else 0.0
    return {"layers": len(table), "mean_coverage": sum(cov.values()) / max(1, len(cov))}


@contextlib.contextmanager
def nvtx(name: str):
    if get_engine_config().nvtx and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class LayerTimer:
    def __init__(self):
        self.ms: dict[int, list[float]] = {}
        self._pending: list[tuple[int, torch.cuda.Event, torch.cuda.Event]] = []

    @contextlib.contextmanager
    def time(self, layer: int):
        if not torch.cuda.is_available() or torch.cuda.is_current_stream_capturing():
            yield
            return
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            self._pending.append((layer, a, b))

    def collect(self) -> None:
        for layer, a, b in self._pending:
            b.synchronize()
            self.ms.setdefault(layer, []).append(a.elapsed_time(b))
        self._pending = []

    def report(self) -> dict[int, float]:
        self.collect()
        return {l: sum(v) / len(v) for l, v in sorted(self.ms.items())}


class StepProfiler:
    """Torch profiler over a window of engine steps (XIAOTU_TORCH_PROFILE=dir[:first:count])."""

    def __init__(self, spec: str):
        parts = spec.split(":")
        self.dir = parts[0]
        self.first = int(parts[1]) if len(parts) > 1 else 2
        self.count = int(parts[2]) if len(parts) > 2 else 3
        self.step = 0
        self.prof = None

    def before_step(self) -> None:
        if self.step == self.first and self.prof is None:
            acts = [torch.profiler.ProfilerActivity.CPU]
            if torch.cuda.is_available():
                acts.append(torch.profiler.ProfilerActivity.CUDA)
            self.prof = torch.profiler.profile(activities=acts)
            self.prof.__enter__()

    def after_step(self) -> None:
        self.step += 1
        if self.prof is not None and self.step >= self.first + self.count:
            self.prof.__exit__(None, None, None)
            os.makedirs(self.dir, exist_ok=True)
            out = os.path.join(self.dir, f"xtu_trace_pid{os.getpid()}.json")
            self.prof.export_chrome_trace(out)
            print(f"[xtu] torch profile written to {out}", file=sys.stderr, flush=True)
            self.prof = None


class Tracer:
    """Per-engine bundle of the enabled hooks (all off by default: zero cost)."""

    def __init__(self, model, ec=None):
        ec = ec or get_engine_config()
        c = model.cfg
        self.routing = (RoutingDump(ec.routing_dump, c.num_layers + len(getattr(model, "mtp", [])),
                                    max(1, c.num_experts), model.device) if ec.routing_dump else None)
        self.timer = LayerTimer() if ec.layer_timing else None
        self.profiler = StepProfiler(ec.torch_profile) if ec.torch_profile else None

    @contextlib.contextmanager
    def layer(self, idx: int):
        with nvtx(f"layer{idx}"):
            if self.timer is not None:
                with self.timer.time(idx):
                    yield
            else:
                yield

    def close(self) -> None:
        if self.routing is not None:
            self.routing.flush()
        if self.profiler is not None and self.profiler.prof is not None:
            self.profiler.count = 0
            self.profiler.after_step()


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="routing dump -> XTUP hot-expert table")
    ap.add_argument("dump")
    ap.add_argument("out")
    ap.add_argument("--per-layer", type=int, default=16)
    a = ap.parse_args(argv)
    print(json.dumps(to_xtup(a.dump, a.out, a.per_layer)))


if __name__ == "__main__":
    main()
