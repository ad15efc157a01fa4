"""Router: scores -> (biased) group-limited top-k -> renormalised, scaled weights.

Covers the scoring functions of the served families: softmax (Mixtral, Qwen),
sigmoid with an ``e_score_correction_bias`` and group-limited selection
(DeepSeek-V3 "noaux_tc", GLM-4.5), and sqrt-softplus (DeepSeek-V4), matching
the options the reference passes to vLLM's ``fused_topk_bias``
(vllm_xiaotu_moe/hybrid_model.py:1877-1890, mixed_experts.py:994-1078).
Selection uses score + bias; the returned weights use the unbiased score.
"""
from __future__ import annotations

import torch

from . import _native as N

SCORING = {"softmax": 0, "sigmoid": 1, "sqrtsoftplus": 2}


def _scores(logits: torch.Tensor, scoring: str) -> torch.Tensor:
    lf = logits.float()
    if scoring == "softmax":
        return torch.softmax(lf, dim=-1)
    if scoring == "sigmoid":
        return torch.sigmoid(lf)
    if scoring == "sqrtsoftplus":
        return torch.sqrt(torch.nn.functional.softplus(lf))
    raise ValueError(scoring)


def router_topk_ref(logits, top_k, scoring="softmax", bias=None, n_group=1, topk_group=1, renorm=True, scale=1.0):
    sc = _scores(logits, scoring)
    sel = sc + (bias.float() if bias is not None else 0.0)
    T, E = sel.shape
    if n_group > 1 and topk_group < n_group:
        g = sel.view(T, n_group, E // n_group)
        gscore = g.topk(2, dim=-1).values.sum(-1)
        keep = gscore.topk(topk_group, dim=-1).indices
        mask = torch.zeros(T, n_group, dtype=torch.bool, device=sel.device)
        mask.scatter_(1, keep, True)
        # experts of dropped groups rank below every kept one but stay selectable (index
        # order), so a top_k above the kept groups' experts still gives distinct experts
        sel = sel.masked_fill(~mask.repeat_interleave(E // n_group, dim=1), torch.finfo(torch.float32).min)
    ids = torch.sort(sel, dim=-1, descending=True, stable=True).indices[:, :top_k]
    w = sc.gather(1, ids)
    if renorm:
        w = w / w.sum(-1, keepdim=True).clamp(min=1e-20)
    return ids.int(), (w * scale).float()


def router_topk(logits: torch.Tensor, top_k: int, scoring: str = "softmax", bias: torch.Tensor | None = None,
                n_group: int = 1, topk_group: int = 1, renorm: bool = True, scale: float = 1.0,
                out_ids: torch.Tensor | None = None, out_w: torch.Tensor | None = None):
    """logits [T, E] fp32 -> (ids int32 [T, K], weights fp32 [T, K])."""
    if not logits.is_cuda:
        return router_topk_ref(logits, top_k, scoring, bias, n_group, topk_group, renorm, scale)
    T, E = logits.shape
    if logits.dtype != torch.float32:
        logits = logits.float()
    assert logits.stride(1) == 1
    ids = out_ids if out_ids is not None else torch.empty(T, top_k, dtype=torch.int32, device=logits.device)
    w = out_w if out_w is not None else torch.empty(T, top_k, dtype=torch.float32, device=logits.device)
    N.call("xtu_router_topk", logits.data_ptr(), N.ptr(bias), T, E, top_k, SCORING[scoring], n_group, topk_group,
           int(renorm), float(scale), ids.data_ptr(), w.data_ptr(), logits.stride(0), N.stream_ptr(logits.device))
    return ids, w


def zipf_bias(num_experts: int, s: float = 1.1, seed: int = 0, strength: float = 1.0) -> torch.Tensor:
    """Seeded per-expert logit bias log(Zipf(s) weight) over a random expert order,
    used by the synthetic benchmarks to create hot experts."""
    g = torch.Generator().manual_seed(seed)
    order = torch.randperm(num_experts, generator=g)
    ranks = torch.empty(num_experts)
    ranks[order] = torch.arange(1, num_experts + 1, dtype=torch.float32)
    w = ranks.pow(-s)
    w = w / w.sum()
    return (strength * torch.log(w * num_experts)).float()
