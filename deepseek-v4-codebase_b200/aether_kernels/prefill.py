"""Chunked prefill against the paged TurboQuant cache (config: several
requests, each a chunk of new query tokens attending to its cached context).

The per-query-row CSA math of aether_2b/modeling.py:591-642: every query
token t scores the visible compressed blocks s < t // compression with the
lightning indexer (modeling.py:609-611), keeps the exact top-k, and attends
to those blocks plus its causal 128-token window with the sink.

``csa_prefill_topk`` runs the indexer on the tcgen05 tensor cores (kernel
csa_prefill_index_kernel): 32 query tokens per CTA against 128-key tiles of
the request's index pages.  ``csa_prefill_attend`` runs the sparse sink
attention of every query token over its top-k blocks and its causal window
on the tcgen05 tensor cores as well (kernel csa_prefill_attend_kernel: one
persistent CTA per SM, S = K q^T and O^T = V^T P from one shared-memory tile
of the token's rows).  ``csa_prefill_chunk`` chains the two.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import _check, _cuda, _stream, rademacher_diag
from .paged import HEAD_DIM, INDEX_DIM, INDEX_HEADS, TurboQuantPagedCache

QUERIES_PER_CTA = 32


@dataclass
class PrefillRequest:
    first_row: int     # row of the request's first query in the stacked query tensors
    num_queries: int   # query tokens in this chunk
    position: int      # absolute position t of the first query token
    nblocks: int       # compressed blocks in the cache (this chunk's own blocks included)


def _plan(requests: Sequence[PrefillRequest], device) -> Tuple[torch.Tensor, torch.Tensor, int]:
    info = torch.tensor([[r.first_row, r.num_queries, r.position, r.nblocks] for r in requests],
                        dtype=torch.int32).reshape(-1, 4)
    tiles = [(i, q) for i, r in enumerate(requests) for q in range(0, r.num_queries, QUERIES_PER_CTA)]
    tl = torch.tensor(tiles, dtype=torch.int32).reshape(-1, 2)
    return info.to(device), tl.to(device), len(tiles)


def csa_prefill_topk(index_q: torch.Tensor, index_weight: torch.Tensor, cache: TurboQuantPagedCache,
                     page_table: torch.Tensor, requests: Sequence[PrefillRequest], compression: int = 4,
                     top_k: int = 256, err: Optional[torch.Tensor] = None,
                     plan: Optional[Tuple[torch.Tensor, torch.Tensor, int]] = None,
                     indexer: str = "exact") -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact top-k blocks per query token.  index_q [Q, 4, 64] fp32,
    index_weight [Q, 4] fp32 raw head weights, page_table [R, max_pages] int32
    (row r for requests[r]).  Returns (keys, ids), each [Q, top_k] int32 (keys
    are order-preserving u32 score bits + 1, reinterpreted), ids ascending,
    padded with key 0 / id -1.

    ``indexer="exact"`` computes the scores exactly (two fp16 limbs of the
    fixed-point rotated query).  ``indexer="fp8"`` computes them on e4m3
    operands (the paper's low-precision indexer): one MMA column per (query,
    head), half the tensor-core K steps; the selection then recalls the exact
    top-k only approximately."""
    _cuda(index_q, "index_q")
    _cuda(index_weight, "index_weight")
    _cuda(page_table, "page_table")
    _check(getattr(cache, "codebook", "uniform") == "uniform", "chunked prefill reads the uniform code format")
    _check(index_q.dtype == torch.float32 and index_weight.dtype == torch.float32,
           "index_q and index_weight must be float32")
    Q = index_q.shape[0]
    _check(tuple(index_q.shape) == (Q, INDEX_HEADS, INDEX_DIM) and tuple(index_weight.shape) == (Q, INDEX_HEADS),
           "index_q must be [Q, 4, 64] and index_weight [Q, 4]")
    _check(page_table.dtype == torch.int32 and page_table.shape[0] >= len(requests), "page_table must be int32 [R, P]")
    _check(cache.idx_pages is not None, "the cache has no indexer stream")
    for r in requests:
        _check(0 <= r.first_row and r.first_row + r.num_queries <= Q, "request rows outside index_q")
        _check(0 <= r.nblocks <= page_table.shape[1] * 64, "request blocks exceed its page-table row")
    dev = index_q.device
    info, tiles, ntiles = plan if plan is not None else _plan(requests, dev)
    keys = torch.zeros(Q, top_k, dtype=torch.int32, device=dev)
    ids = torch.full((Q, top_k), -1, dtype=torch.int32, device=dev)
    _check(indexer in ("exact", "fp8"), f"indexer must be 'exact' or 'fp8', got {indexer!r}")
    entry = "aether_csa_prefill_topk" if indexer == "exact" else "aether_csa_prefill_topk_fp8"
    _lib.call(entry, index_q.data_ptr(), index_weight.data_ptr(), cache.idx_pages.data_ptr(),
              page_table.data_ptr(), page_table.shape[1], cache.num_pages, info.data_ptr(), tiles.data_ptr(), ntiles,
              int(compression), rademacher_diag(INDEX_DIM, cache.seed, dev).data_ptr(), cache.bits, int(top_k),
              keys.data_ptr(), ids.data_ptr(), None if err is None else err.data_ptr(), _stream(dev))
    return keys, ids


def query_rows(requests: Sequence[PrefillRequest], compression: int, window: int, window_first_row: Sequence[int],
               device) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per query token: (page-table row, visible blocks, first window row,
    window length) for a flat window buffer where request r's raw window
    rows start at window_first_row[r] with the row of position
    ``position - window + 1``."""
    q_row, vis, wrow, wlen = [], [], [], []
    for r, (req, w0) in enumerate(zip(requests, window_first_row)):
        for i in range(req.num_queries):
            t = req.position + i
            q_row.append(r)
            vis.append(min(req.nblocks, t // compression))
            n = min(window, t + 1)
            wlen.append(n)
            wrow.append(w0 + i + (window - n))
    return (torch.tensor(q_row, dtype=torch.int32, device=device), torch.tensor(vis, dtype=torch.int32, device=device),
            torch.tensor(wrow, dtype=torch.int64, device=device), torch.tensor(wlen, dtype=torch.int32, device=device))


def csa_prefill_attend(q: torch.Tensor, sink: torch.Tensor, window: torch.Tensor, win_row: torch.Tensor,
                       window_len: torch.Tensor, cache: TurboQuantPagedCache, page_table: torch.Tensor,
                       q_row: torch.Tensor, nblocks: torch.Tensor, cand_keys: torch.Tensor, cand_ids: torch.Tensor,
                       softmax_scale: float, out: Optional[torch.Tensor] = None,
                       indices: Optional[torch.Tensor] = None,
                       err: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Sparse sink attention of each query token over its candidate blocks
    plus its window.  q [Q, H, 128] bf16, sink [H] fp32, window [rows, 128]
    bf16 (flat), win_row [Q] int64, window_len [Q] int32 (<= 128), q_row [Q]
    int32 page-table row, nblocks [Q] int32 visible blocks, cand_keys /
    cand_ids [Q, top_k] from ``csa_prefill_topk``.  Returns (out [Q, H, 128]
    bf16 before the inverse output RoPE, attended ids [Q, top_k])."""
    for t, nm in ((q, "q"), (sink, "sink"), (window, "window"), (win_row, "win_row"), (window_len, "window_len"),
                  (page_table, "page_table"), (q_row, "q_row"), (nblocks, "nblocks"), (cand_keys, "cand_keys"),
                  (cand_ids, "cand_ids")):
        _cuda(t, nm)
    Q, H, D = q.shape
    _check(D == HEAD_DIM and q.dtype == torch.bfloat16 and window.dtype == torch.bfloat16,
           "q [Q, H, 128] and window [rows, 128] must be bfloat16")
    _check(win_row.dtype == torch.int64 and q_row.dtype == torch.int32 and nblocks.dtype == torch.int32
           and window_len.dtype == torch.int32, "win_row int64; q_row, nblocks, window_len int32")
    top_k = cand_ids.shape[1]
    dev = q.device
    if out is None:
        out = torch.empty(Q, H, D, dtype=torch.bfloat16, device=dev)
    if indices is None:
        indices = torch.empty(Q, top_k, dtype=torch.int32, device=dev)
    _lib.call("aether_csa_prefill_attend", q.data_ptr(), sink.data_ptr(), window.data_ptr(), win_row.data_ptr(),
              window_len.data_ptr(), cache.kv_pages.data_ptr(), page_table.data_ptr(), page_table.shape[1],
              cache.num_pages, q_row.data_ptr(), nblocks.data_ptr(), page_table.shape[1] * 64,
              rademacher_diag(HEAD_DIM, cache.seed, dev).data_ptr(), cand_keys.data_ptr(), cand_ids.data_ptr(),
              cand_ids.shape[1], Q, H, cache.bits, int(top_k), float(softmax_scale), out.data_ptr(),
              indices.data_ptr(), None if err is None else err.data_ptr(), _stream(dev))
    return out, indices


def csa_prefill_chunk(q, index_q, index_weight, sink, window, window_first_row: Sequence[int],
                      cache: TurboQuantPagedCache, page_table, requests: Sequence[PrefillRequest],
                      softmax_scale: float, compression: int = 4, top_k: int = 256, err=None,
                      indexer: str = "exact"):
    """Indexer top-k then attention for every query token of the chunks.
    Returns (out [Q, H, 128] bf16, selected block ids [Q, top_k])."""
    keys, ids = csa_prefill_topk(index_q, index_weight, cache, page_table, requests, compression, top_k, err,
                                 indexer=indexer)
    q_row, vis, wrow, wlen = query_rows(requests, compression, 128, window_first_row, q.device)
    return csa_prefill_attend(q, sink, window, wrow, wlen, cache, page_table, q_row, vis, keys, ids, softmax_scale,
                              err=err)
