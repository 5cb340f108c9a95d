"""CPU restatements of the reference extension's dense ops.  TEST ORACLE ONLY.

  * ``sparse_attention``  -- PytorchAttentionBackend.sparse_attention,
                             aether_pipeline/serving.py:99-130 (gather by
                             index, logits * scale, max incl. sink, exp,
                             normalise with exp(sink), weighted V sum)
  * ``dense_index_topk``  -- canonical indexer aether_2b/modeling.py:609-615
                             with (score desc, index asc) ordering
  * ``hca_compress``      -- aether_2b/serving.py:495-498 in fp32:
                             softmax over the window per channel, weighted sum
"""
from __future__ import annotations

import torch


def sparse_attention(q, kv, topk_indices, sink, softmax_scale):
    q = q.float()
    kv = kv.float()
    sink = sink.float()
    B, T, H, D = q.shape
    S = kv.shape[1]
    idx = topk_indices.long()
    valid = (idx >= 0) & (idx < S)
    safe = idx.clamp(0, max(S - 1, 0))
    keys = kv[:, :, 0][torch.arange(B).view(B, 1, 1), safe]     # [B, T, K, D]
    vals = kv[:, :, 1][torch.arange(B).view(B, 1, 1), safe]
    logits = torch.einsum("bthd,btkd->bthk", q, keys) * softmax_scale
    logits = logits.masked_fill(~valid[:, :, None, :], float("-inf"))
    if sink.numel() == 1:
        sk = sink.reshape(1, 1, 1, 1)
    else:
        sk = sink.view(1, 1, -1, 1)
    mx = torch.maximum(logits.max(dim=-1, keepdim=True).values, sk)
    e = torch.exp(logits - mx)
    w = e / (e.sum(dim=-1, keepdim=True) + torch.exp(sk - mx))
    return torch.einsum("bthk,btkd->bthd", w, vals)


def dense_index_topk(index_q, index_kv, index_weight, k):
    s = torch.einsum("bhc,bsc->bhs", index_q.float(), index_kv.float())
    s = (torch.relu(s) * torch.nn.functional.softplus(index_weight.float()).unsqueeze(-1)).sum(dim=1)
    return torch.sort(s, dim=-1, descending=True, stable=True).indices[:, :k], s


def dense_index_scores64(index_q, index_kv, index_weight):
    """fp64 indexer scores [B, S] and each row's score magnitude bound
    sum_h softplus(w_h) max_s sum_c |q_hc k_sc| (the near-tie scale)."""
    q, kv, w = index_q.double(), index_kv.double(), torch.nn.functional.softplus(index_weight.double())
    s = (torch.relu(torch.einsum("bhc,bsc->bhs", q, kv)) * w.unsqueeze(-1)).sum(dim=1)
    mag = (torch.einsum("bhc,bsc->bhs", q.abs(), kv.abs()) * w.unsqueeze(-1)).sum(dim=1).amax(dim=-1)
    return s, mag


def hca_compress(buffer_c, buffer_z):
    w = torch.softmax(buffer_z.float(), dim=1)
    return (w * buffer_c.float()).sum(dim=1)
