"""Seeded synthetic decode batches with the shapes and value distributions of
the benchmark configurations (no datasets or checkpoints are involved):

  q, compressed K (=V), index q / k, window ~ N(0, 1); raw head weights
  ~ N(0, 1) (softplus applied by the indexer); sink ~ N(0, 1); compressed
  entries rotated by RoPE at their end-of-block positions i*m + m - 1
  (aether_2b/modeling.py:477-481), window rows and the query at their token
  positions; pages allocated in random order.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from .paged import HEAD_DIM, INDEX_DIM, INDEX_HEADS, PAGE, TurboQuantPagedCache
from .rope import RopeConfig, apply_rope, rope_attention_scale


@dataclass
class DecodeBatch:
    kind: str                     # "csa" or "hca"
    q: torch.Tensor               # [B, H, 128] bf16
    index_q: Optional[torch.Tensor]       # [B, 4, 64] fp32
    index_weight: Optional[torch.Tensor]  # [B, 4] fp32
    sink: torch.Tensor            # [H] fp32
    window: torch.Tensor          # [B, W, 128] bf16
    window_len: torch.Tensor      # [B] int32
    cache: TurboQuantPagedCache
    page_table: torch.Tensor      # [B, max_pages] int32
    nblocks: torch.Tensor         # [B] int32
    tokens: List[int]             # token count per sequence (decode position)
    softmax_scale: float
    top_k: int
    bits: int
    # raw (unquantized, post-RoPE) compressed entries, kept only when asked
    raw_kv: Optional[List[torch.Tensor]] = None
    raw_index: Optional[List[torch.Tensor]] = None


def make_decode_batch(
    kind: str,
    batch: int,
    ctx_lo: int,
    ctx_hi: int,
    bits: int,
    compression: int,
    heads: int = 12,
    window: int = 128,
    top_k: int = 256,
    seed: int = 0,
    device="cuda",
    rope: Optional[RopeConfig] = None,
    cache: Optional[TurboQuantPagedCache] = None,
    gen_device: str = "cpu",
    keep_raw: bool = False,
    max_blocks: Optional[int] = None,
) -> DecodeBatch:
    """Build one synthetic decode batch.  Context lengths (tokens) are drawn
    uniformly from [ctx_lo, ctx_hi]; nblocks = tokens // compression.  With
    ``cache`` given, pages are allocated from it (so several batches can
    share one pool); otherwise a pool just large enough is created."""
    rope = rope or RopeConfig()
    dev = torch.device(device)
    g = torch.Generator(device=gen_device)
    g.manual_seed(seed)
    gd = torch.device(gen_device)

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=gd)

    if ctx_hi > ctx_lo:
        toks = (ctx_lo + torch.randint(0, ctx_hi - ctx_lo + 1, (batch,), generator=g, device=gd)).tolist()
    else:
        toks = [ctx_lo] * batch
    nbs = [t // compression for t in toks]
    if max_blocks is not None:
        nbs = [min(n, max_blocks) for n in nbs]
    max_nb = max(nbs) if nbs else 0
    max_pages = max(1, (max_nb + PAGE - 1) // PAGE)
    need_pages = sum((n + PAGE - 1) // PAGE for n in nbs)
    if cache is None:
        cache = TurboQuantPagedCache(max(need_pages, 1), bits, dev, with_index=(kind == "csa"))
    pg = torch.Generator()
    pg.manual_seed(seed + 7919)
    page_table = torch.zeros(batch, max_pages, dtype=torch.int32)
    seq_pages = []
    for b, n in enumerate(nbs):
        pages = cache.alloc_pages((n + PAGE - 1) // PAGE, generator=pg)
        seq_pages.append(pages)
        if pages:
            page_table[b, : len(pages)] = torch.tensor(pages, dtype=torch.int32)
    page_table = page_table.to(dev)

    raw_kv, raw_index = ([], []) if keep_raw else (None, None)
    for b, n in enumerate(nbs):
        if n == 0:
            if keep_raw:
                raw_kv.append(torch.empty(0, HEAD_DIM))
                raw_index.append(torch.empty(0, INDEX_DIM))
            continue
        pos = torch.arange(n, device=gd) * compression + (compression - 1)
        kv = apply_rope(randn(n, HEAD_DIM), pos, rope).to(dev)
        idx = randn(n, INDEX_DIM).to(dev) if kind == "csa" else None
        pt = page_table[b: b + 1]
        start = torch.zeros(1, dtype=torch.int32, device=dev)
        cache.write(pt, start, kv.unsqueeze(0), None if idx is None else idx.unsqueeze(0))
        if keep_raw:
            raw_kv.append(kv.cpu())
            raw_index.append(idx.cpu() if idx is not None else torch.empty(0, INDEX_DIM))

    pos_q = torch.tensor(toks, device=gd, dtype=torch.float32)
    q = apply_rope(randn(batch, heads, HEAD_DIM).unsqueeze(1), pos_q.view(batch, 1), rope).squeeze(1)
    win = randn(batch, window, HEAD_DIM)
    wpos = pos_q.view(batch, 1) - (window - 1) + torch.arange(window, device=gd).view(1, window)
    win = apply_rope(win, wpos, rope)
    wlen = torch.tensor([min(window, t + 1) for t in toks], dtype=torch.int32)
    # rows are oldest first; a short window keeps its valid rows at the front
    for b, t in enumerate(toks):
        if t + 1 < window:
            win[b, : t + 1] = win[b, window - (t + 1):].clone()
            win[b, t + 1:] = 0
    index_q = randn(batch, INDEX_HEADS, INDEX_DIM).to(dev) if kind == "csa" else None
    index_w = randn(batch, INDEX_HEADS).to(dev) if kind == "csa" else None
    sink = randn(heads).to(dev)
    return DecodeBatch(
        kind=kind,
        q=q.to(dev, torch.bfloat16).contiguous(),
        index_q=index_q,
        index_weight=index_w,
        sink=sink,
        window=win.to(dev, torch.bfloat16).contiguous(),
        window_len=wlen.to(dev),
        cache=cache,
        page_table=page_table,
        nblocks=torch.tensor(nbs, dtype=torch.int32, device=dev),
        tokens=toks,
        softmax_scale=HEAD_DIM ** -0.5 * rope_attention_scale(rope),
        top_k=top_k,
        bits=bits,
        raw_kv=raw_kv,
        raw_index=raw_index,
    )
