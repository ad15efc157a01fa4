"""Hot-expert (PIN) table tooling: routing dumps -> coverage report, held-out hit rate,
XTUP tables and fixed-size seed tables (the reference's scripts/expert_profile.py:1-191
and scripts/make_seed_pin_table.py:1-104).

    python -m vllm_xtu_moe_b200.tiering.pin_tools profile dump.json [--slots 8,16,32] [--folds 10]
    python -m vllm_xtu_moe_b200.tiering.pin_tools table dump.json out.xtup --per-layer 16
    python -m vllm_xtu_moe_b200.tiering.pin_tools seed out.xtup --model glm-4.5-air --budget-gib 20 [--dump d.json]

* Coverage (in-sample, an upper bound): the share of a layer's routed pairs that its N
  most frequent experts receive.
* Held-out hit rate (the honest figure): the dump's windows are dealt into ``folds``
  folds; each fold is predicted by the per-layer top-N of the other folds and scored on
  its own pairs.  Computed per layer and summed, never on a pool of all layers (a
  cross-layer pool mixes experts that share an id but not their weights).
* Seed tables: the same number of slots in every MoE layer, sized from a memory budget
  with the slot formula of the pool itself (``host.expert_slot_bytes``: weights plus
  block scales for the layer's format), filled with each layer's hottest experts when a
  dump is given, else its first experts; the pool's route-driven swap-in replaces cold
  seeds at run time.
"""
from __future__ import annotations

import argparse
import json
import sys

from .host import expert_slot_bytes
from .policy import save_pin_table, table_from_counts


def _top(counts: list[int], n: int) -> set[int]:
    order = sorted(range(len(counts)), key=lambda e: (-counts[e], e))
    return {e for e in order[:n] if counts[e] > 0}


def coverage(counts: dict[int, list[int]], slots: int) -> dict:
    """In-sample top-N coverage per layer and over all layers' pairs."""
    per, hit, tot = {}, 0, 0
    for l, c in counts.items():
        t = sum(c)
        h = sum(c[e] for e in _top(c, slots))
        per[l] = h / t if t else 0.0
        hit += h
        tot += t
    return {"slots": slots, "coverage": hit / tot if tot else 0.0, "per_layer": per}


def heldout_hit_rate(windows: list[dict[int, list[int]]], slots: int, folds: int = 10) -> float:
    """k-fold held-out hit rate of a per-layer top-N table (NaN with fewer windows than folds)."""
    n = len(windows)
    if n < folds or folds < 2:
        return float("nan")
    layers = sorted({l for w in windows for l in w})
    hits = tot = 0
    for f in range(folds):
        test = windows[f::folds]
        for l in layers:
            train = None
            for i, w in enumerate(windows):
                if i % folds == f or l not in w:
                    continue
                train = list(w[l]) if train is None else [a + b for a, b in zip(train, w[l])]
            top = _top(train, slots) if train is not None else set()
            for w in test:
                c = w.get(l)
                if c is None:
                    continue
                tot += sum(c)
                hits += sum(c[e] for e in top)
    return hits / tot if tot else float("nan")


def lru_hit_rate(windows: list[dict[int, list[int]]], cap: int) -> float:
    """Session-level hit rate of a global LRU cache of ``cap`` (layer, expert) slots
    replayed over the windows in order (a lower-bound probe of routing locality)."""
    from collections import OrderedDict
    cache: OrderedDict = OrderedDict()
    hits = tot = 0
    for w in windows:
        for l in sorted(w):
            for e, c in enumerate(w[l]):
                if c <= 0:
                    continue
                tot += c
                key = (l, e)
                if key in cache:
                    hits += c
                    cache.move_to_end(key)
                else:                  # the window's first pair misses and loads; the rest hit
                    if cap <= 0:
                        continue
                    hits += c - 1
                    if len(cache) >= cap:
                        cache.popitem(last=False)
                    cache[key] = None
    return hits / tot if tot else float("nan")


def slots_for_budget(budget_gib: float, fmt: str, hidden: int, inter: int, moe_layers: int) -> int:
    """Slots per layer that fit a pool budget (every MoE layer gets the same count)."""
    per = expert_slot_bytes(fmt, hidden, inter)
    return max(0, int(budget_gib * (1 << 30) // (per * max(1, moe_layers))))


def seed_table(moe_layers: list[int], num_experts: int, slots: int,
               counts: dict[int, list[int]] | None = None) -> dict[int, list[int]]:
    """Every listed layer gets ``slots`` experts: its hottest from ``counts`` (topped up
    with the lowest ids not chosen), else experts 0..slots-1."""
    slots = min(slots, num_experts)
    out = {}
    for l in moe_layers:
        pick = []
        if counts is not None and l in counts:
            c = counts[l]
            pick = [e for e in sorted(range(len(c)), key=lambda e: (-c[e], e)) if c[e] > 0][:slots]
        rest = [e for e in range(num_experts) if e not in set(pick)]
        out[l] = pick + rest[:slots - len(pick)]
    return out


def profile(dump: str, slots: list[int], folds: int = 10) -> dict:
    from ..utils.trace import load_dump, load_windows
    E, counts = load_dump(dump)
    wins = load_windows(dump)
    rep = {"experts": E, "layers": len(counts), "windows": len(wins), "pairs": sum(sum(c) for c in counts.values()),
           "by_slots": []}
    for n in slots:
        cov = coverage(counts, n)
        rep["by_slots"].append({"slots": n, "coverage_in_sample": round(cov["coverage"], 4),
                                "hit_rate_heldout": round(heldout_hit_rate(wins, n, folds), 4),
                                "hit_rate_lru_global": round(lru_hit_rate(wins, n * max(1, len(counts))), 4)})
    return rep


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("profile", help="coverage and held-out hit rate of top-N tables")
    p.add_argument("dump")
    p.add_argument("--slots", default="8,16,32,64")
    p.add_argument("--folds", type=int, default=10)
    t = sub.add_parser("table", help="XTUP table of each layer's N hottest experts")
    t.add_argument("dump")
    t.add_argument("out")
    t.add_argument("--per-layer", type=int, default=16)
    s = sub.add_parser("seed", help="fixed-size seed table sized from a memory budget")
    s.add_argument("out")
    s.add_argument("--model", default="glm-4.5-air")
    s.add_argument("--budget-gib", type=float, default=None)
    s.add_argument("--slots-per-layer", type=int, default=None)
    s.add_argument("--dump", default=None)
    a = ap.parse_args(argv)
    if a.cmd == "profile":
        print(json.dumps(profile(a.dump, [int(x) for x in a.slots.split(",")], a.folds)))
        return
    if a.cmd == "table":
        from ..utils.trace import load_dump
        E, counts = load_dump(a.dump)
        table = table_from_counts(counts, a.per_layer)
        save_pin_table(a.out, table, E)
        print(json.dumps({"layers": len(table), **{k: v for k, v in coverage(counts, a.per_layer).items()
                                                   if k != "per_layer"}}))
        return
    from ..models.config import get_preset
    cfg = get_preset(a.model)
    layers = [i for i in range(cfg.num_layers) if cfg.is_moe_layer(i)]
    per_slot = expert_slot_bytes(cfg.expert_fmt, cfg.hidden_size, cfg.moe_intermediate)
    if a.slots_per_layer is None and a.budget_gib is None:
        print("give --budget-gib or --slots-per-layer", file=sys.stderr)
        raise SystemExit(2)
    n = a.slots_per_layer if a.slots_per_layer is not None else slots_for_budget(
        a.budget_gib, cfg.expert_fmt, cfg.hidden_size, cfg.moe_intermediate, len(layers))
    counts = None
    if a.dump:
        from ..utils.trace import load_dump
        _, counts = load_dump(a.dump)
    table = seed_table(layers, cfg.num_experts, n, counts)
    save_pin_table(a.out, table, cfg.num_experts)
    print(json.dumps({"layers": len(layers), "slots_per_layer": n, "slot_bytes": per_slot,
                      "pool_gib": round(n * len(layers) * per_slot / (1 << 30), 3)}))


if __name__ == "__main__":
    main()
