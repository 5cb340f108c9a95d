"""CPU restatement of the chunked-prefill indexer selection.  TEST ORACLE ONLY.

Follows aether_2b/modeling.py:591-615 of the reference for query tokens that
come after a cached prefix: query token t scores the compressed blocks
s < t // compression (the causal block mask of :612-614, with the cache
holding every block formed so far) with the canonical indexer
sum_h softplus(w_h) * relu(q_h . k_s) (:609-611) over keys decoded from the
paged TurboQuant cache, and keeps the exact top min(top_k, visible) with
ties to the lower block index.  Near-tie rows are flagged as in
``oracle.decode``.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import turboquant as tq
from .decode import gather_pages, index_scores, topk_stable


def prefill_topk(index_q, index_weight, idx_codes, idx_scale, page_table, requests: Sequence[Tuple[int, int, int, int]],
                 bits: int, top_k: int, compression: int = 4, seed: int = 42,
                 tie_tol: float = 1e-5, rows: Optional[Sequence[int]] = None) -> Tuple[List[torch.Tensor], List[bool]]:
    """requests: (first_row, num_queries, position of query 0, nblocks) per
    request.  Returns per query row (in request order) the selected block ids
    ascending, and a near-tie flag; with ``rows`` (query rows to check, in
    ascending order) only those rows, in that order."""
    sels, ties = [], []
    want = None if rows is None else set(int(x) for x in rows)
    for r, (row0, nq, pos0, nblk) in enumerate(requests):
        if want is not None and not any(row0 <= x < row0 + nq for x in want):
            continue
        keys = tq.decode(gather_pages(idx_codes, page_table[r], nblk),
                         gather_pages(idx_scale, page_table[r], nblk).unsqueeze(-1), bits, seed)
        for i in range(nq):
            if want is not None and row0 + i not in want:
                continue
            vis = min(nblk, (pos0 + i) // compression)
            k = min(top_k, vis)
            if vis == 0:
                sels.append(torch.empty(0, dtype=torch.long))
                ties.append(False)
                continue
            iq, iw = index_q[row0 + i].float(), index_weight[row0 + i].float()
            s32 = index_scores(iq, iw, keys[:vis])
            sels.append(torch.sort(topk_stable(s32, k)).values)
            tie = False
            if vis > k:
                kd = keys[:vis].double()
                s64 = index_scores(iq.double(), iw.double(), kd)
                srt = torch.sort(s64, descending=True).values
                mag = (iq.double().abs() @ kd.abs().T)
                mag = (mag * torch.nn.functional.softplus(iw.double()).unsqueeze(-1)).sum(0).max()
                tie = bool(srt[k - 1] - srt[k] <= tie_tol * float(mag))
            ties.append(tie)
    return sels, ties
