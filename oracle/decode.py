"""CPU restatement of one CSA / HCA decode step over a paged TurboQuant cache.
TEST ORACLE ONLY (see the package docstring).

Follows the reference's fp32 torch path:
  * page gather        -- aether_2b/serving.py:486-493 (pages concatenated in
                          table order), entry i at page i // 64, slot i % 64
  * dequant            -- PolarQuant.decode, aether_2b/turbo_quant.py:168-211
                          (``oracle.turboquant.decode``)
  * indexer score      -- aether_2b/modeling.py:609-611:
                          sum_h softplus(w_h) * relu(q_h . k_s)   (einsum in fp32)
  * top-k              -- modeling.py:615 / serving.py:620-621 with an explicit
                          stable order (score desc, index asc) in place of
                          torch.topk's unspecified tie order
  * sparse sink attn   -- aether_pipeline/serving.py:99-130 (fp32), sources =
                          [selected compressed ; window] as in serving.py:624,
                          K == V (serving.py:52-53)
  * HCA                -- serving.py:507-522: every visible block + window

Near-tie rows: the kernel computes index scores in another (exact-integer,
rotated-domain) order, so a row whose fp64 scores at ranks k and k+1 differ
by less than ``tie_tol`` * sum_h w_h sum_c |q_hc k_c| may legitimately pick
a different block; such rows are reported, not failed.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from . import turboquant as tq

PAGE = 64


def gather_pages(pool: torch.Tensor, table_row: torch.Tensor, n: int) -> torch.Tensor:
    """Rows 0..n-1 of one sequence from a [P, 64, ...] pool."""
    if n == 0:
        return pool.new_empty(0, *pool.shape[2:])
    npg = (n + PAGE - 1) // PAGE
    pages = pool[table_row[:npg].long()]
    return pages.reshape(npg * PAGE, *pool.shape[2:])[:n]


def index_scores(iq: torch.Tensor, iw: torch.Tensor, keys: torch.Tensor) -> torch.Tensor:
    """fp32 canonical indexer (modeling.py:609-611). iq [IH, IC], iw [IH], keys [S, IC]."""
    s = torch.einsum("hc,sc->hs", iq, keys)
    return (torch.relu(s) * torch.nn.functional.softplus(iw).unsqueeze(-1)).sum(dim=0)


def topk_stable(scores: torch.Tensor, k: int) -> torch.Tensor:
    """Indices of the k largest scores ordered by (score desc, index asc)."""
    # a stable descending sort keeps the lower index first among equal scores
    return torch.sort(scores, descending=True, stable=True).indices[:k]


def sink_attention(q: torch.Tensor, src: torch.Tensor, sink: torch.Tensor, scale: float) -> torch.Tensor:
    """q [H, D], src [S, D] (K == V), sink [H] -> [H, D]; aether_pipeline/serving.py:99-130."""
    if src.shape[0] == 0:
        return torch.zeros_like(q)
    logits = (q @ src.T) * scale
    mx = torch.maximum(logits.max(dim=-1, keepdim=True).values, sink.view(-1, 1))
    e = torch.exp(logits - mx)
    w = e / (e.sum(dim=-1, keepdim=True) + torch.exp(sink.view(-1, 1) - mx))
    return w @ src


@dataclass
class DecodeResult:
    out: torch.Tensor                 # [B, H, D] fp32
    selected: List[torch.Tensor]      # per row: selected block indices, ascending
    near_tie: List[bool]              # per row: ranks k / k+1 within the fp32 noise band


def decode_step(kind: str, q, index_q, index_weight, sink, window, window_len, idx_codes, idx_scale, kv_codes,
                kv_scale, page_table, nblocks, bits: int, top_k: int, softmax_scale: float, seed: int = 42,
                tie_tol: float = 1e-5, use_selection: Optional[List[torch.Tensor]] = None,
                classify_ties: bool = True, levels: Optional[torch.Tensor] = None) -> DecodeResult:
    """All tensors on the CPU.  ``use_selection`` replaces the oracle's top-k
    by a given per-row selection (to check attention on a near-tie row);
    ``classify_ties=False`` skips the fp64 near-tie bookkeeping (timing);
    ``levels`` decodes a cache in the Lloyd-Max level format
    (``oracle.turboquant.decode_lut``) instead of the uniform one."""
    B, H, D = q.shape

    def dec(codes, scale):
        if levels is None:
            return tq.decode(codes, scale, bits, seed)
        return tq.decode_lut(codes, scale, bits, levels, seed)

    outs, sels, ties = [], [], []
    for b in range(B):
        nb = int(nblocks[b])
        wl = int(window_len[b])
        table = page_table[b]
        main = dec(gather_pages(kv_codes, table, nb), gather_pages(kv_scale, table, nb).unsqueeze(-1))
        tie = False
        if kind == "csa":
            keys = dec(gather_pages(idx_codes, table, nb), gather_pages(idx_scale, table, nb).unsqueeze(-1))
            k = min(top_k, nb)
            if use_selection is not None:
                sel = use_selection[b].long()
            elif nb > 0:
                s32 = index_scores(index_q[b].float(), index_weight[b].float(), keys)
                sel = torch.sort(topk_stable(s32, k)).values
                if nb > k and classify_ties:
                    s64 = index_scores(index_q[b].double(), index_weight[b].double(), keys.double())
                    srt = torch.sort(s64, descending=True).values
                    mag = (index_q[b].double().abs() @ keys.double().abs().T)
                    mag = (mag * torch.nn.functional.softplus(index_weight[b].double()).unsqueeze(-1)).sum(0).max()
                    tie = bool(srt[k - 1] - srt[k] <= tie_tol * float(mag))
            else:
                sel = torch.empty(0, dtype=torch.long)
            chosen = main[sel]
        else:
            sel = torch.arange(nb)
            chosen = main
        src = torch.cat([chosen, window[b, :wl].float()], dim=0)
        outs.append(sink_attention(q[b].float(), src, sink.float(), softmax_scale))
        sels.append(sel)
        ties.append(tie)
    return DecodeResult(torch.stack(outs), sels, ties)
