"""DeepSeek sparse attention (DSA) ops: lightning-indexer scores, per-query top-k token
selection, and MLA attention over the selected latent rows (``csrc/cuda/dsa.cu`` + the MLA
latent decode kernel).

Per query row t of sequence b at position p:

    I[t, j] = sum_h w[t, h] * relu(q[t, h] . k[j])          j = 0 .. p  (index keys k of b)
    S_t     = the index_topk positions of largest I[t, .]  (all of 0 .. p when p < index_topk)
    o[t]    = MLA attention of q[t] over the latent cache rows of S_t

The selection is returned as flat rows of the paged latent cache (``block_table[b][j // 64] *
64 + j % 64``) in position order.  Attention gathers each query's rows into a contiguous
run of 64-row blocks and runs the latent decode kernel with one pseudo-sequence per query
(every selected row is visible: all positions are <= p).  CPU restatements of the three
steps serve as the test oracle.
"""
from __future__ import annotations

import torch

from . import _native as N
from .attention import AttnMetadata, choose_splits, paged_attention, paged_attention_ref

BLOCK = 64


def seq_of_rows(q_start: torch.Tensor, T: int) -> torch.Tensor:
    """[T] int32 sequence index of every query row (device op, graph-capturable)."""
    rows = torch.arange(T, dtype=q_start.dtype, device=q_start.device)
    return (torch.searchsorted(q_start, rows, right=True) - 1).to(torch.int32)


def index_scores(q: torch.Tensor, w: torch.Tensor, k_cache: torch.Tensor, meta: AttnMetadata, seq: torch.Tensor,
                 ld: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """q [T, nh, 128] bf16, w [T, nh] fp32 (scales folded in), k_cache [blocks, 1, 64, 128]
    -> scores [T, ld] fp32 (entries past a row's position are not written)."""
    T, nh, d = q.shape
    scores = out if out is not None else torch.empty(T, ld, dtype=torch.float32, device=q.device)
    if q.is_cuda:
        assert q.stride(2) == 1 and q.stride(1) == d and d == 128 and w.is_contiguous()
        N.call("xtu_dsa_index_scores", q.data_ptr(), q.stride(0), nh, w.data_ptr(), k_cache.data_ptr(),
               meta.block_table.data_ptr(), meta.block_table.stride(0), seq.data_ptr(), meta.positions.data_ptr(),
               T, ld, k_cache.shape[0], scores.data_ptr(), scores.stride(0), N.status_buffer(q.device).data_ptr(),
               N.stream_ptr(q.device))
        return scores
    kc = k_cache[:, 0].reshape(-1, d).float()
    for t in range(T):
        b, p = int(seq[t]), int(meta.positions[t])
        nb = p // BLOCK + 1
        rows = (meta.block_table[b, :nb].long()[:, None] * BLOCK + torch.arange(BLOCK)).reshape(-1)[:p + 1]
        s = torch.relu(q[t].float() @ kc[rows].t())                   # [nh, p+1]
        scores[t, :p + 1] = (w[t].float()[:, None] * s).sum(0)
    return scores


def topk_rows(scores: torch.Tensor, meta: AttnMetadata, seq: torch.Tensor, k: int,
              rows: torch.Tensor | None = None, lens: torch.Tensor | None = None):
    """-> (rows [T, k] int32 flat latent-cache rows in position order, lens [T] int32)."""
    T = scores.shape[0]
    d = scores.device
    rows = rows if rows is not None else torch.empty(T, k, dtype=torch.int32, device=d)
    lens = lens if lens is not None else torch.empty(T, dtype=torch.int32, device=d)
    if scores.is_cuda:
        N.call("xtu_dsa_topk", scores.data_ptr(), scores.stride(0), meta.positions.data_ptr(), seq.data_ptr(),
               meta.block_table.data_ptr(), meta.block_table.stride(0), T, k, rows.data_ptr(), lens.data_ptr(),
               N.stream_ptr(d))
        return rows, lens
    for t in range(T):
        b, p = int(seq[t]), int(meta.positions[t])
        n = min(p + 1, k)
        sel = torch.arange(p + 1) if p + 1 <= k else torch.topk(scores[t, :p + 1], k).indices.sort().values
        rows[t, :n] = (meta.block_table[b, sel // BLOCK].long() * BLOCK + sel % BLOCK).to(torch.int32)
        lens[t] = n
    return rows, lens


class SparsePlan:
    """Static buffers of the sparse attention of T query rows (graph-capturable): the gather
    target and the pseudo-sequence metadata (query t owns blocks t * kb .. t * kb + kb - 1).
    The gather target starts zeroed: the attention kernel reads whole 64-row blocks and
    multiplies the rows past a query's selection by a zero probability, which must not meet
    a NaN bit pattern (later calls leave finite latent rows there)."""

    def __init__(self, T: int, k: int, width: int, device):
        self.kb = (k + BLOCK - 1) // BLOCK
        self.T = T
        self.scratch = torch.zeros(T * self.kb, 1, BLOCK, width, dtype=torch.bfloat16, device=device)
        self.q_start = torch.arange(T + 1, dtype=torch.int32, device=device)
        self.bt = torch.arange(T * self.kb, dtype=torch.int32, device=device).view(T, self.kb)
        self.zeros = torch.zeros(T, dtype=torch.int32, device=device)


def sparse_mla(q: torch.Tensor, k_cache: torch.Tensor, rows: torch.Tensor, lens: torch.Tensor, scale: float,
               v_dim: int, plan: SparsePlan | None = None) -> torch.Tensor:
    """q [T, nh, D] bf16 (absorbed MLA queries), k_cache [blocks, 1, 64, D] latent cache ->
    o [T, nh, v_dim] over each row's selected cache rows (rows / lens from ``topk_rows``)."""
    T, nh, D = q.shape
    k = rows.shape[1]
    flat = k_cache.view(-1, D)
    if not q.is_cuda:
        out = torch.empty(T, nh, v_dim, dtype=q.dtype)
        for t in range(T):
            kv = flat[rows[t, :int(lens[t])].long()].float()               # [n, D]
            s = (q[t].float() @ kv.t()) * scale                            # [nh, n]
            out[t] = (torch.softmax(s, -1) @ kv[:, :v_dim]).to(q.dtype)
        return out
    plan = plan if plan is not None and plan.T == T else SparsePlan(T, k, D, q.device)
    N.call("xtu_dsa_gather", k_cache.data_ptr(), D, flat.shape[0], rows.data_ptr(), lens.data_ptr(), T, k,
           plan.kb * BLOCK, plan.scratch.data_ptr(), N.status_buffer(q.device).data_ptr(), N.stream_ptr(q.device))
    meta = AttnMetadata(num_seqs=T, q_start=plan.q_start, kv_len=lens, block_table=plan.bt,
                        slot_mapping=plan.zeros, positions=plan.zeros, max_q_len=1, max_kv_len=plan.kb * BLOCK,
                        is_decode=True)
    meta.num_splits = choose_splits(T, 1, plan.kb * BLOCK)
    return paged_attention(q, plan.scratch, None, meta, scale, v_dim=v_dim)


def sparse_mla_dense_ref(q: torch.Tensor, k_cache: torch.Tensor, rows: torch.Tensor, lens: torch.Tensor,
                         scale: float, v_dim: int) -> torch.Tensor:
    """The same attention through the dense paged-attention oracle (test helper)."""
    T, nh, D = q.shape
    flat = k_cache.view(-1, D).cpu().float()
    out = torch.empty(T, nh, v_dim, dtype=torch.float32)
    for t in range(T):
        n = int(lens[t])
        nb = (n + BLOCK - 1) // BLOCK
        kc = torch.zeros(nb * BLOCK, D)
        kc[:n] = flat[rows[t, :n].long().cpu()]
        m = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, 1]), kv_len=torch.tensor([n]),
                         block_table=torch.arange(nb, dtype=torch.int32)[None], slot_mapping=torch.zeros(1),
                         positions=torch.zeros(1), max_q_len=1, max_kv_len=n, is_decode=True,
                         q_start_host=[0, 1], kv_len_host=[n])
        out[t] = paged_attention_ref(q[t:t + 1].float().cpu(), kc.view(nb, 1, BLOCK, D), None, m, scale,
                                     v_dim=v_dim)[0]
    return out
