"""Chunked prefill against the paged TurboQuant cache (config: several
requests, each a chunk of new query tokens attending to its cached context).

The per-query-row CSA math of aether_2b/modeling.py:591-642: every query
token t scores the visible compressed blocks s < t // compression with the
lightning indexer (modeling.py:609-611), keeps the exact top-k, and attends
to those blocks plus its causal 128-token window with the sink.

``csa_prefill_topk`` runs the indexer on the tcgen05 tensor cores (kernel
csa_prefill_index_kernel): 32 query tokens per CTA against 128-key tiles of
the request's index pages.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import _check, _cuda, _stream, rademacher_diag
from .paged import INDEX_DIM, INDEX_HEADS, TurboQuantPagedCache

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
                     plan: Optional[Tuple[torch.Tensor, torch.Tensor, int]] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact top-k blocks per query token.  index_q [Q, 4, 64] fp32,
    index_weight [Q, 4] fp32 raw head weights, page_table [R, max_pages] int32
    (row r for requests[r]).  Returns (keys, ids), each [Q, top_k] int32 (keys
    are order-preserving u32 score bits + 1, reinterpreted), ids ascending,
    padded with key 0 / id -1."""
    _cuda(index_q, "index_q")
    _cuda(index_weight, "index_weight")
    _cuda(page_table, "page_table")
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
    _lib.call("aether_csa_prefill_topk", index_q.data_ptr(), index_weight.data_ptr(), cache.idx_pages.data_ptr(),
              page_table.data_ptr(), page_table.shape[1], cache.num_pages, info.data_ptr(), tiles.data_ptr(), ntiles,
              int(compression), rademacher_diag(INDEX_DIM, cache.seed, dev).data_ptr(), cache.bits, int(top_k),
              keys.data_ptr(), ids.data_ptr(), None if err is None else err.data_ptr(), _stream(dev))
    return keys, ids
