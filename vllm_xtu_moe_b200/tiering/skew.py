"""Skewed expert popularity for benchmarks of random-init models.

A random router spreads tokens almost evenly over the experts, which real MoE checkpoints
do not: a few experts per layer take most of the traffic, and the hot-expert pool and the
PIN tables exist for that.  The tiered benchmark configurations therefore bias the router
with a seeded Zipf(s = 1.1) term per expert (as :func:`..ops.router.zipf_bias` does for
the single-layer sweeps).

:func:`zipf_order` draws, per MoE layer, the popularity order of the experts (a seeded
permutation: expert ``order[r]`` has Zipf rank r).  :func:`apply_zipf_router_bias` adds
``scale * (log p_r - log p_0)`` (p the Zipf(s) pmf over E ranks) to each layer's
selection bias (the e_score_correction_bias slot: it moves which experts are picked, not
their weights).  ``scale`` is set per layer so that the hottest quarter of the experts
receives the Zipf(s) share of the routed pairs; the bias then competes with, rather than
replaces, the token-dependent part of the routing.
"""
from __future__ import annotations

import torch


def zipf_order(num_experts: int, layers: list[int], seed: int = 0) -> dict[int, list[int]]:
    """Per layer, the experts in decreasing popularity (seeded permutation)."""
    out = {}
    for l in layers:
        g = torch.Generator().manual_seed(seed * 1000003 + l)
        out[l] = torch.randperm(num_experts, generator=g).tolist()
    return out


def zipf_log_pmf(num_experts: int, s: float) -> torch.Tensor:
    """log p_r - log p_0 of Zipf(s) over ranks 0 .. E-1 (0 for the hottest rank)."""
    r = torch.arange(1, num_experts + 1, dtype=torch.float64)
    return (-s * torch.log(r)).float()


def zipf_share(num_experts: int, top: int, s: float) -> float:
    """Share of Zipf(s) mass on the `top` most popular of `num_experts` ranks."""
    w = torch.arange(1, num_experts + 1, dtype=torch.float64).pow(-s)
    return float(w[:top].sum() / w.sum())


@torch.no_grad()
def apply_zipf_router_bias(model, order: dict[int, list[int]], s: float = 1.1, samples: int = 512,
                           seed: int = 0) -> dict[int, float]:
    """Bias every MoE layer of ``model`` (main and MTP layers) whose index is in ``order``;
    returns the per-layer scale used.

    The scale is calibrated per layer on unit-variance router inputs (the router reads an
    RMS-normalised hidden state) by bisection, so that the routed pairs landing on the
    hottest quarter of the experts match the Zipf(s) share of that quarter."""
    from ..models.layers import MoEBlock
    from ..ops.router import router_topk_ref
    blocks = [l.mlp for l in model.layers] + [m.layer.mlp for m in getattr(model, "mtp", [])]
    scales = {}
    g = torch.Generator().manual_seed(seed)
    for b in blocks:
        if not isinstance(b, MoEBlock) or b.layer_idx not in order:
            continue
        c = b.cfg
        E, H = b.gate.shape
        x = torch.randn(samples, H, generator=g)
        logits = x @ b.gate.float().cpu().t()
        base = b.gate_bias.float().cpu() if b.gate_bias is not None else torch.zeros(E)
        lp = torch.empty(E)
        lp[torch.tensor(order[b.layer_idx][:E])] = zipf_log_pmf(E, s)
        hot = torch.tensor(order[b.layer_idx][: max(1, E // 4)])
        target = zipf_share(E, max(1, E // 4), s)

        def share(scale):
            ids, _ = router_topk_ref(logits, c.top_k, c.scoring, base + scale * lp, c.n_group, c.topk_group)
            return torch.isin(ids, hot).float().mean().item()

        lo, hi = 0.0, 1.0
        while share(hi) < target and hi < 1e4:
            lo, hi = hi, hi * 4
        for _ in range(24):
            mid = 0.5 * (lo + hi)
            lo, hi = (mid, hi) if share(mid) < target else (lo, mid)
        scale = 0.5 * (lo + hi)
        bias = (scale * lp).to(b.gate.device)
        if b.gate_bias is not None:
            b.gate_bias.add_(bias.to(b.gate_bias.dtype))
        else:
            b.gate_bias = bias
        scales[b.layer_idx] = scale
    return scales
