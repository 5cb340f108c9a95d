"""Op wrappers with the reference's signatures (aether_kernels/sparse_attention.py:8-83),
plus the fused paged-cache entry points of this package."""
from __future__ import annotations

import torch

from .loader import load_aether_cuda_kernels
from .paged import csa_decode_paged, hca_decode_paged  # noqa: F401  (fused entry points)


def sparse_sink_attention(
    q: torch.Tensor,
    kv: torch.Tensor,
    topk_indices: torch.Tensor,
    sink: torch.Tensor,
    softmax_scale: float,
) -> torch.Tensor:
    """softmax([q.k_j * scale]_j U sink) . V over the gathered sources.

    q [B, T, H, D], kv [B, S, 2, D] (K, V), topk_indices [B, T, K] int32/int64
    (entries outside [0, S) are skipped), sink scalar or [H] in q's dtype."""
    ext = load_aether_cuda_kernels()
    return ext.sparse_sink_attention(q, kv, topk_indices, sink, float(softmax_scale))


def tiled_prefill_attention(
    q: torch.Tensor,
    kv: torch.Tensor,
    sink: torch.Tensor,
    softmax_scale: float,
    tile_size: int = 256,
) -> torch.Tensor:
    """Attention of every target token over all S sources with the sink
    counted once in the denominator.  q [B, T, H, D], kv [B, S, 2, D]."""
    ext = load_aether_cuda_kernels()
    return ext.tiled_prefill_attention(q.contiguous(), kv.contiguous(), sink.contiguous(), float(softmax_scale),
                                       int(tile_size))


def csa_indexer_topk(
    index_q: torch.Tensor,
    index_kv: torch.Tensor,
    index_weight: torch.Tensor,
    k: int,
) -> torch.Tensor:
    """Lightning indexer: score[s] = sum_h softplus(w_h) * relu(q_h . k_s);
    returns the exact top-k source indices [B, k] int64 ordered by
    (score desc, index asc).  index_q [B, IH, IC], index_kv [B, S, IC],
    index_weight [B, IH] raw weights, all float32."""
    ext = load_aether_cuda_kernels()
    return ext.csa_indexer_topk(index_q.float().contiguous(), index_kv.float().contiguous(),
                                index_weight.float().contiguous(), int(k))


def hca_compress(buffer_c: torch.Tensor, buffer_z: torch.Tensor) -> torch.Tensor:
    """Softmax-weighted reduction of one HCA window: buffer_c, buffer_z
    [B, M, D] -> [B, D] (softmax over M per channel)."""
    ext = load_aether_cuda_kernels()
    return ext.hca_compress(buffer_c.contiguous(), buffer_z.contiguous())
