"""Token sampling for requests that do not decode greedily.

The model step always produces the greedy token of every logits row (an argmax kernel,
inside the decode CUDA graph).  Rows whose request asks for temperature > 0 are then
re-drawn here from the same logits, on the device: temperature scaling, top-k, top-p
(nucleus) filtering, and one draw from the request's own generator, seeded from
``SamplingParams.seed`` when given, so a seeded request reproduces its tokens.
"""
from __future__ import annotations

import torch


def _generator(req, device: torch.device) -> torch.Generator:
    g = getattr(req, "_generator", None)
    if g is None or g.device != device:
        g = torch.Generator(device=device)
        seed = req.params.seed
        g.manual_seed(int(seed) if seed is not None else int(torch.randint(0, 2 ** 62, (1,)).item()))
        req._generator = g
    return g


def filtered_probs(logits: torch.Tensor, temperature: float, top_k: int = 0, top_p: float = 1.0) -> torch.Tensor:
    """Sampling distribution of one row of logits [V] (fp32 probabilities)."""
    x = logits.float() / max(temperature, 1e-6)
    if 0 < top_k < x.numel():
        kth = torch.topk(x, top_k).values[-1]
        x = torch.where(x < kth, torch.full_like(x, float("-inf")), x)
    p = torch.softmax(x, dim=-1)
    if top_p < 1.0:
        sp, idx = torch.sort(p, descending=True)
        cum = torch.cumsum(sp, dim=-1)
        drop = (cum - sp) > top_p                # keep the smallest prefix reaching top_p
        sp = torch.where(drop, torch.zeros_like(sp), sp)
        p = torch.zeros_like(p).scatter_(0, idx, sp)
        p = p / p.sum()
    return p


def needs_sampling(reqs) -> bool:
    return any(r.params.temperature > 0.0 for r in reqs)


def sample_rows(logits: torch.Tensor, reqs: list, greedy: torch.Tensor) -> torch.Tensor:
    """Tokens for logits rows [n, V] of requests ``reqs`` (one per row): greedy rows keep
    ``greedy``, the others are drawn from their filtered distribution."""
    out = greedy.clone()
    for i, r in enumerate(reqs):
        sp = r.params
        if sp.temperature <= 0.0:
            continue
        p = filtered_probs(logits[i], sp.temperature, sp.top_k, sp.top_p)
        out[i] = torch.multinomial(p, 1, generator=_generator(r, logits.device)).to(out.dtype)[0]
    return out


def wants_logprobs(reqs) -> int:
    """Largest number of alternatives any request asks for, or -1 when none wants logprobs."""
    ks = [r.params.logprobs for r in reqs if r.params.logprobs is not None]
    return max(ks) if ks else -1


def row_logprobs(logits: torch.Tensor, tokens: torch.Tensor, k: int) -> list:
    """Per row: (log-probability of the chosen token under the model's distribution,
    {token: log-probability} of the k most likely tokens)."""
    lp = torch.log_softmax(logits.float(), dim=-1)
    chosen = lp.gather(1, tokens.long().view(-1, 1)).view(-1).tolist()
    out = []
    if k > 0:
        vals, idx = torch.topk(lp, k, dim=-1)
        vals, idx = vals.tolist(), idx.tolist()
    for i, c in enumerate(chosen):
        out.append((c, dict(zip(idx[i], vals[i])) if k > 0 else {}))
    return out
