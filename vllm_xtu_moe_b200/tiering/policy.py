"""Hot-expert pool: routing-table files and the swap policy.

XTUP v1 routing table (file format kept identical to the reference so existing
tables load; vllm_xiaotu_moe/expert_pool.py:119-136):
    header  <4sIIII>  magic b"XTUP", version 1, n_layers, n_experts, n_entries
    entries <HH>      (layer, expert), most frequently routed first

``plan_swap`` decides which resident experts to evict and which hot experts to load
after a window of routing counts.  Its rules follow the reference policy
(expert_pool.py:60-113), restated here:
  1. victims are the coldest residents, ordered by (count, pool order); ties go to
     the oldest resident, or to the newest with ``preserve_oldest`` (prefill windows);
  2. candidates are non-resident experts with count >= min_hits, hottest first;
  3. hysteresis: a candidate replaces its victim only if count > victim * (1 + hyst);
  4. rate limit: at most maxswap (default max(1, nslots // 4)) swaps per window;
  5. an empty pool never swaps; evicted and loaded sets never overlap.
"""
from __future__ import annotations

import struct
from pathlib import Path

_HDR = "<4sIIII"
_ENT = "<HH"


def load_pin_table(path: str | Path) -> dict[int, list[int]]:
    """layer -> experts, most frequent first.  A damaged table (wrong magic or version, a
    header or entry count that runs past the file, a layer or expert outside the header's
    ranges, an expert listed twice for one layer) raises ValueError naming the problem,
    so a bad file never places the wrong experts silently."""
    buf = Path(path).read_bytes()
    hsz, esz = struct.calcsize(_HDR), struct.calcsize(_ENT)
    if len(buf) < hsz:
        raise ValueError(f"XTUP table {path}: {len(buf)} bytes, shorter than its header")
    magic, ver, n_layers, n_experts, n_ent = struct.unpack_from(_HDR, buf, 0)
    if magic != b"XTUP" or ver != 1:
        raise ValueError(f"not an XTUP v1 table: {magic!r} v{ver}")
    if len(buf) < hsz + esz * n_ent:
        raise ValueError(f"XTUP table {path}: {n_ent} entries announced, {(len(buf) - hsz) // esz} present")
    out: dict[int, list[int]] = {}
    for i in range(n_ent):
        layer, expert = struct.unpack_from(_ENT, buf, hsz + esz * i)
        if layer >= n_layers or expert >= n_experts:
            raise ValueError(f"XTUP table {path}: entry {i} (layer {layer}, expert {expert}) outside "
                             f"{n_layers} layers x {n_experts} experts")
        lst = out.setdefault(int(layer), [])
        if expert in lst:
            raise ValueError(f"XTUP table {path}: expert {expert} listed twice for layer {layer}")
        lst.append(int(expert))
    return out


def save_pin_table(path: str | Path, table: dict[int, list[int]], n_experts: int) -> None:
    entries = [(l, e) for l in sorted(table) for e in table[l]]
    n_layers = (max(table) + 1) if table else 0
    with open(path, "wb") as f:
        f.write(struct.pack(_HDR, b"XTUP", 1, n_layers, n_experts, len(entries)))
        for l, e in entries:
            f.write(struct.pack(_ENT, l, e))


def table_from_counts(counts: dict[int, list[int]], per_layer: int) -> dict[int, list[int]]:
    """Routing counts (layer -> per-expert counts) -> the per_layer hottest experts of each layer."""
    out = {}
    for layer, c in counts.items():
        order = sorted(range(len(c)), key=lambda e: (-c[e], e))
        out[layer] = [e for e in order[:per_layer] if c[e] > 0]
    return out


def plan_swap(resident: list[int], counts: dict[int, int], nslots: int, *, hyst: float = 0.25, maxswap: int = 0,
              min_hits: int = 1, preserve_oldest: bool = False) -> tuple[list[int], list[int]]:
    """-> (evict, load): experts leaving the pool and experts entering it, pairwise."""
    if nslots <= 0 or not resident:
        return [], []
    res = list(resident)
    k = maxswap if maxswap > 0 else max(1, nslots // 4)
    if preserve_oldest:
        order = sorted(range(len(res)), key=lambda i: (counts.get(res[i], 0), -i))
    else:
        order = sorted(range(len(res)), key=lambda i: (counts.get(res[i], 0), i))
    cold = order[:k]
    in_res = set(res)
    cands = sorted(((e, c) for e, c in counts.items() if e not in in_res and c >= min_hits),
                   key=lambda kv: (-kv[1], kv[0]))[:k]
    evict, load = [], []
    for i, (e, c) in enumerate(cands):
        if i >= len(cold):
            break
        victim = res[cold[i]]
        if c > counts.get(victim, 0) * (1.0 + hyst):
            evict.append(victim)
            load.append(e)
    assert not (set(evict) & set(load))
    assert all(counts.get(v, 0) <= counts.get(l, 0) for v, l in zip(evict, load))
    return evict, load


def pool_hits(counts: dict[int, int] | list[int], experts: list[int]) -> tuple[int, int]:
    """(routed pairs that went to a pooled expert, all routed pairs) for per-expert counts
    (the reference's PIN hit-rate windows, vllm_xiaotu_moe/mixed_experts.py:3020-3100)."""
    if isinstance(counts, dict):
        items = counts.items()
    else:
        items = enumerate(counts)
    pooled = set(experts)
    hit = tot = 0
    for e, c in items:
        tot += int(c)
        if e in pooled:
            hit += int(c)
    return hit, tot
