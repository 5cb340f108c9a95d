"""Batched decode rounds of a model's CSA / HCA attention layers over the
paged TurboQuant cache.

The reference's serving engine steps one request at a time
(aether_2b/scheduler.py:357-426) and, per layer and token, de-quantizes the
whole compressed cache, scores it with torch ops, gathers, concatenates the
window and calls the attention backend (``_attention_step_csa``,
aether_2b/serving.py:597-654; ``_attention_step_hca``, :507-538).
``DecodeRound`` keeps that data flow for a whole batch and replaces its
attention core with the fused kernels: per layer one
``csa_decode_paged`` (indexer, exact top-k, sparse sink attention, inverse
output RoPE) or ``hca_decode_paged`` launch for every sequence of the round,
reading quantized pages in place.

What it keeps per layer and sequence, as the reference's serving state does:
  * the sliding window (the last ``window`` entries including the current
    one, oldest first);
  * the open compression block: CSA's a / b halves of the main and index
    streams (plus the previous block's b half for the overlap), HCA's
    (c, z + bias[slot]) rows;
  * the token count, from which the visible blocks are ``pos // m``.
When a block closes, ``TurboQuantPagedCache.emit_csa`` / ``emit_hca`` pool it
(softmax gate, RoPE at the block start for CSA and the block end for HCA,
RMSNorm, TurboQuant encode) straight into the sequence's next page slot.

The caller supplies what the model's projections produce for the step (q
after its norm, the index query and raw head weights, the window entry, the
compression inputs); ``rows`` selects the sequences taking part, so requests
can join and leave a round at different positions.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from .paged import HEAD_DIM, INDEX_DIM, PAGE, TurboQuantPagedCache, csa_decode_paged, csa_workspace_bytes, \
    hca_decode_paged
from .rope import RopeConfig, apply_rope, get_rope_freqs, rope_attention_scale


@dataclass
class AttentionLayerSpec:
    """One attention layer's fixed parameters (aether_2b/modeling.py
    CSAAttention / HCAAttention): the per-head sink, the compressed entries'
    RMSNorm weight and eps, and the emit biases."""

    kind: str                                   # "csa" or "hca"
    sink: torch.Tensor                          # [H] fp32
    norm_weight: torch.Tensor                   # [128]
    norm_eps: float = 1e-6
    bias_a: Optional[torch.Tensor] = None       # CSA [m, 128]
    bias_b: Optional[torch.Tensor] = None
    index_bias_a: Optional[torch.Tensor] = None  # CSA [m, 64]
    index_bias_b: Optional[torch.Tensor] = None
    bias: Optional[torch.Tensor] = None         # HCA [m_h, 128]


class DecodeRound:
    """Decode state and fused attention for ``batch`` sequences of a model."""

    def __init__(self, layers: Sequence[AttentionLayerSpec], batch: int, max_tokens: int, *, bits: int = 4,
                 csa_compression: int = 4, hca_compression: int = 128, window: int = 128, top_k: int = 256,
                 rope: Optional[RopeConfig] = None, device="cuda", seed: int = 42):
        self.dev = torch.device(device)
        self.B, self.W, self.top_k = batch, window, top_k
        self.m = {"csa": csa_compression, "hca": hca_compression}
        self.rope = rope or RopeConfig()
        self.inv_freq = get_rope_freqs(self.rope, device=self.dev).float().contiguous()
        self.scale = HEAD_DIM ** -0.5 * rope_attention_scale(self.rope)
        self.layers: List[Dict[str, object]] = []
        f32 = dict(dtype=torch.float32, device=self.dev)
        for spec in layers:
            if spec.kind not in ("csa", "hca"):
                raise ValueError(f"layer kind must be 'csa' or 'hca', got {spec.kind!r}")
            m = self.m[spec.kind]
            max_blocks = max_tokens // m
            pages = max(1, (max_blocks + PAGE - 1) // PAGE)
            cache = TurboQuantPagedCache(batch * pages, bits, self.dev, with_index=spec.kind == "csa", seed=seed)
            table = torch.tensor([cache.alloc_pages(pages) for _ in range(batch)], dtype=torch.int32,
                                 device=self.dev)
            st: Dict[str, object] = dict(spec=spec, cache=cache, table=table, pos=torch.zeros(batch, dtype=torch.long),
                                         win=torch.zeros(batch, window, HEAD_DIM, dtype=torch.bfloat16,
                                                         device=self.dev))
            if spec.kind == "csa":
                for nm, d in (("a_c", HEAD_DIM), ("a_z", HEAD_DIM), ("b_c", HEAD_DIM), ("b_z", HEAD_DIM),
                              ("pb_c", HEAD_DIM), ("pb_z", HEAD_DIM), ("ia_c", INDEX_DIM), ("ia_z", INDEX_DIM),
                              ("ib_c", INDEX_DIM), ("ib_z", INDEX_DIM), ("pib_c", INDEX_DIM), ("pib_z", INDEX_DIM)):
                    st[nm] = torch.zeros(batch, m, d, **f32)
                st["has_prev"] = torch.zeros(batch, dtype=torch.int32, device=self.dev)
                st["ws"] = torch.zeros(csa_workspace_bytes(batch, pages * PAGE), dtype=torch.uint8, device=self.dev)
            else:
                st["c"] = torch.zeros(batch, m, HEAD_DIM, **f32)
                st["z"] = torch.zeros(batch, m, HEAD_DIM, **f32)
            self.layers.append(st)

    # ---------------------------------------------------------------- state
    def positions(self, layer: int) -> torch.Tensor:
        """Token count of every sequence at ``layer`` (the next position)."""
        return self.layers[layer]["pos"].clone()

    def _rows(self, rows) -> torch.Tensor:
        if rows is None:
            return torch.arange(self.B)
        return torch.as_tensor(rows, dtype=torch.long).flatten()

    def _push_window(self, st, rows: torch.Tensor, entry: torch.Tensor) -> torch.Tensor:
        """Append the step's window entry (the reference keeps the last W-1
        entries plus the current one); returns the window lengths [R] int32."""
        pos = st["pos"][rows]
        win = st["win"]
        e = entry.to(self.dev, torch.bfloat16)
        full = pos >= self.W
        if bool(full.any()):
            fr = rows[full].to(self.dev)
            win[fr] = torch.cat([win[fr, 1:], e[full.to(self.dev)].unsqueeze(1)], dim=1)
        nf = ~full
        if bool(nf.any()):
            win[rows[nf].to(self.dev), pos[nf].to(self.dev)] = e[nf.to(self.dev)]
        return torch.clamp(pos + 1, max=self.W).to(torch.int32)

    # ----------------------------------------------------------------- CSA
    def step_csa(self, layer: int, q: torch.Tensor, index_q: torch.Tensor, index_weight: torch.Tensor,
                 window_entry: torch.Tensor, kv_a: torch.Tensor, z_a: torch.Tensor, kv_b: torch.Tensor,
                 z_b: torch.Tensor, index_kv_a: torch.Tensor, index_z_a: torch.Tensor, index_kv_b: torch.Tensor,
                 index_z_b: torch.Tensor, rows=None, err: Optional[torch.Tensor] = None):
        """One decode step of a CSA layer for ``rows`` (default: all).  Inputs
        have one leading row per sequence: q [R, H, 128], index_q [R, 4, 64],
        index_weight [R, 4] (raw, softplus in-kernel), window_entry [R, 128],
        kv_*/z_* [R, 128], index_kv_*/index_z_* [R, 64].  Returns the attention
        output with the inverse output RoPE applied [R, H, 128] bf16 and the
        selected block ids [R, top_k] (ascending, -1 padded)."""
        st = self.layers[layer]
        spec: AttentionLayerSpec = st["spec"]
        if spec.kind != "csa":
            raise ValueError(f"layer {layer} is an HCA layer")
        rows = self._rows(rows)
        r = rows.to(self.dev)
        m = self.m["csa"]
        pos = st["pos"][rows]
        wl = self._push_window(st, rows, window_entry)
        visible = (pos // m).to(torch.int32)
        cache: TurboQuantPagedCache = st["cache"]
        out, sel = csa_decode_paged(q.to(self.dev, torch.bfloat16).contiguous(), index_q.to(self.dev).float().contiguous(),
                                    index_weight.to(self.dev).float().contiguous(), spec.sink.to(self.dev).float(),
                                    st["win"][r].contiguous(), wl.to(self.dev), cache, st["table"][r].contiguous(),
                                    visible.to(self.dev), self.scale, top_k=self.top_k, err=err, workspace=st["ws"],
                                    rope_positions=pos.to(self.dev, torch.int32), rope_inv_freq=self.inv_freq)
        slot = (pos % m).to(self.dev)
        for nm, x in (("a_c", kv_a), ("a_z", z_a), ("b_c", kv_b), ("b_z", z_b), ("ia_c", index_kv_a),
                      ("ia_z", index_z_a), ("ib_c", index_kv_b), ("ib_z", index_z_b)):
            st[nm][r, slot] = x.to(self.dev).float()
        st["pos"][rows] += 1
        closing = ((pos + 1) % m) == 0
        if bool(closing.any()):
            e = r[closing.to(self.dev)]
            epos = pos[closing]
            slot_pos = ((epos + 1) // m - 1).to(self.dev, torch.int32)
            start = (epos - (m - 1)).to(self.dev, torch.int32)  # RoPE at the block's first token
            main = (st["a_c"][e], st["a_z"][e], spec.bias_a.to(self.dev).float(), st["pb_c"][e], st["pb_z"][e],
                    spec.bias_b.to(self.dev).float())
            index = (st["ia_c"][e], st["ia_z"][e], spec.index_bias_a.to(self.dev).float(), st["pib_c"][e],
                     st["pib_z"][e], spec.index_bias_b.to(self.dev).float())
            cache.emit_csa(st["table"][e].contiguous(), slot_pos, main, index, st["has_prev"][e].contiguous(), start,
                           self.inv_freq, spec.norm_weight.to(self.dev).float(), spec.norm_eps, err=err)
            # the closing block's b half overlaps the next block
            st["pb_c"][e], st["pb_z"][e] = st["b_c"][e], st["b_z"][e]
            st["pib_c"][e], st["pib_z"][e] = st["ib_c"][e], st["ib_z"][e]
            st["has_prev"][e] = 1
        return out, sel

    # ----------------------------------------------------------------- HCA
    def step_hca(self, layer: int, q: torch.Tensor, window_entry: torch.Tensor, kv: torch.Tensor, z: torch.Tensor,
                 rows=None, err: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step of an HCA layer: q [R, H, 128], window_entry
        [R, 128], kv = kv_proj(x) and z = z_proj(x) [R, 128] (the slot bias is
        added here).  Returns the attention output with the inverse output
        RoPE applied [R, H, 128] bf16."""
        st = self.layers[layer]
        spec: AttentionLayerSpec = st["spec"]
        if spec.kind != "hca":
            raise ValueError(f"layer {layer} is a CSA layer")
        rows = self._rows(rows)
        r = rows.to(self.dev)
        m = self.m["hca"]
        pos = st["pos"][rows]
        wl = self._push_window(st, rows, window_entry)
        visible = (pos // m).to(torch.int32)
        cache: TurboQuantPagedCache = st["cache"]
        out = hca_decode_paged(q.to(self.dev, torch.bfloat16).contiguous(), spec.sink.to(self.dev).float(),
                               st["win"][r].contiguous(), wl.to(self.dev), cache, st["table"][r].contiguous(),
                               visible.to(self.dev), self.scale, err=err)
        # inverse output RoPE (aether_2b/serving.py:469-472)
        out = apply_rope(out.unsqueeze(1), (-pos).to(self.dev).view(-1, 1), self.rope).squeeze(1)
        slot = (pos % m).to(self.dev)
        st["c"][r, slot] = kv.to(self.dev).float()
        st["z"][r, slot] = z.to(self.dev).float() + spec.bias.to(self.dev).float()[slot]
        st["pos"][rows] += 1
        closing = ((pos + 1) % m) == 0
        if bool(closing.any()):
            e = r[closing.to(self.dev)]
            epos = pos[closing]
            slot_pos = ((epos + 1) // m - 1).to(self.dev, torch.int32)
            cache.emit_hca(st["table"][e].contiguous(), slot_pos, st["c"][e], st["z"][e],
                           epos.to(self.dev, torch.int32), self.inv_freq, spec.norm_weight.to(self.dev).float(),
                           spec.norm_eps, err=err)
        return out
