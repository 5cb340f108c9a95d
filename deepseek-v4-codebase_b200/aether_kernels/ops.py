"""Torch-tensor front end of the C-ABI kernels.

Each function checks its tensors the way the reference extension's
``bindings.cpp`` does (CUDA, contiguous, shapes; ``RuntimeError`` on
failure), allocates outputs with ``torch.empty`` on the input's device, and
launches on the current CUDA stream.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _cuda(t: torch.Tensor, name: str) -> None:
    _check(t.is_cuda, f"{name} must be a CUDA tensor")
    _check(t.is_contiguous(), f"{name} must be contiguous")


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(dev: torch.device) -> int:
    """cudaStream_t of the current stream on ``dev`` (the raw accessor when
    torch has it: the Stream object path costs microseconds per call)."""
    if _RAW_STREAM is not None:
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        return _RAW_STREAM(idx)
    return torch.cuda.current_stream(dev).cuda_stream


def _dt(t: torch.Tensor, name: str) -> int:
    _check(t.dtype in _DTYPE_CODE, f"{name}: unsupported dtype {t.dtype}")
    return _DTYPE_CODE[t.dtype]


# ----------------------------------------------------------------- rotation
_DIAG_CACHE: Dict[Tuple[int, int, str], torch.Tensor] = {}


def rademacher_diag(d: int, seed: int, device: torch.device) -> torch.Tensor:
    """Fixed +-1 diagonal of TurboQuant (aether_2b/turbo_quant.py:111-121):
    a CPU ``torch.Generator`` seeded ``seed * 10007 + d``; +1 where
    ``torch.rand(d) > 0.5``.  Host-side parameter setup, cached per device."""
    key = (d, seed, str(device))
    t = _DIAG_CACHE.get(key)
    if t is None:
        g = torch.Generator()
        g.manual_seed(seed * 10007 + d)
        r = torch.rand(d, generator=g)
        t = torch.where(r > 0.5, torch.ones(d), -torch.ones(d)).to(device)
        _DIAG_CACHE[key] = t
    return t


# --------------------------------------------------------------- TurboQuant
def tq_encode(x: torch.Tensor, bits: int, seed: int = 42) -> Tuple[torch.Tensor, torch.Tensor]:
    d = x.shape[-1]
    _cuda(x, "x")
    lead = x.shape[:-1]
    rows = x.numel() // d if d else 0
    codes = torch.empty(*lead, d if bits == 8 else d // 2, dtype=torch.int8 if bits == 8 else torch.uint8,
                        device=x.device)
    scale = torch.empty(*lead, 1, dtype=torch.float32, device=x.device)
    diag = rademacher_diag(d, seed, x.device)
    _lib.call("aether_tq_encode", x.data_ptr(), _dt(x, "x"), rows, d, bits, diag.data_ptr(), codes.data_ptr(),
              scale.data_ptr(), None, _stream(x.device))
    return codes, scale


def tq_encode_into_pages(x: torch.Tensor, bits: int, page_table: torch.Tensor, start_pos: torch.Tensor,
                         page_pool: torch.Tensor, seed: int = 42, err: Optional[torch.Tensor] = None) -> None:
    """Encode x [B, n, d] and write entry i of sequence b to logical position
    start_pos[b] + i of that sequence's pages: page page_table[b, pos // 64],
    slot pos % 64 of ``page_pool`` [P, 64 * row_bytes + 256] (64 code rows
    followed by 64 fp32 scales per page)."""
    _cuda(x, "x")
    _check(x.dim() == 3, "x must have shape [B, n, D]")
    B, n, d = x.shape
    for t, nm in ((page_table, "page_table"), (start_pos, "start_pos"), (page_pool, "page_pool")):
        _cuda(t, nm)
    _check(page_table.dtype == torch.int32 and start_pos.dtype == torch.int32, "page tables must be int32")
    rb = d * bits // 8
    _check(page_pool.dtype == torch.uint8 and page_pool.dim() == 2 and page_pool.shape[1] == 64 * rb + 256,
           "page_pool must be uint8 [P, 64 * row_bytes + 256]")
    diag = rademacher_diag(d, seed, x.device)
    _lib.call("aether_tq_encode_into_pages", x.data_ptr(), _dt(x, "x"), B, n, d, bits, diag.data_ptr(),
              page_table.data_ptr(), page_table.shape[1], start_pos.data_ptr(), page_pool.shape[0],
              page_pool.data_ptr(), None if err is None else err.data_ptr(), _stream(x.device))


def compress_emit(c0: torch.Tensor, z0: torch.Tensor, bias0: Optional[torch.Tensor] = None,
                  c1: Optional[torch.Tensor] = None, z1: Optional[torch.Tensor] = None,
                  bias1: Optional[torch.Tensor] = None, has_seg1: Optional[torch.Tensor] = None,
                  positions: Optional[torch.Tensor] = None, inv_freq: Optional[torch.Tensor] = None,
                  norm_weight: Optional[torch.Tensor] = None, norm_eps: float = 1e-6, bits: int = 8,
                  page_table: Optional[torch.Tensor] = None, slot_pos: Optional[torch.Tensor] = None,
                  page_pool: Optional[torch.Tensor] = None, seed: int = 42, want_out: bool = True,
                  err: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Fused compress-on-emit for B finishing blocks of one stream.

    ``entry = RMSNorm(RoPE(sum_r softmax_r(z_r + bias_r) * c_r))`` per channel
    over the rows of segment 0 (c0 / z0 [B, m, d]) and, where has_seg1[b],
    segment 1 (c1 / z1 [B, m1, d], CSA's previous-block half), as
    aether_2b/serving.py:495-505 (HCA) and :540-575 (CSA main: RoPE + norm;
    CSA index: neither).  RoPE applies when ``inv_freq`` is given (rope_dim =
    2 * len(inv_freq)); RMSNorm when ``norm_weight`` is given.  With
    ``page_pool`` the entry is TurboQuant-encoded into slot ``slot_pos[b]``
    of sequence b's pages.  Returns the fp32 entry [B, d] when ``want_out``."""
    _cuda(c0, "c0")
    _cuda(z0, "z0")
    _check(c0.dim() == 3 and z0.shape == c0.shape, "c0 and z0 must have the same shape [B, m, d]")
    B, m0, d = c0.shape
    _check(c0.dtype == z0.dtype, "c and z must share a dtype")
    dev = c0.device

    def f32(t, shape, nm):
        if t is None:
            return None
        _cuda(t, nm)
        _check(t.dtype == torch.float32 and tuple(t.shape) == tuple(shape), f"{nm} must be float32 {list(shape)}")
        return t.contiguous()

    bias0 = f32(bias0, (m0, d), "bias0")
    m1 = 0
    if c1 is not None:
        _cuda(c1, "c1")
        _cuda(z1, "z1")
        _check(c1.dim() == 3 and z1.shape == c1.shape and c1.shape[0] == B and c1.shape[2] == d
               and c1.dtype == c0.dtype, "c1 / z1 must be [B, m1, d] in c0's dtype")
        m1 = c1.shape[1]
        bias1 = f32(bias1, (m1, d), "bias1")
        if has_seg1 is not None:
            _cuda(has_seg1, "has_seg1")
            _check(has_seg1.dtype == torch.int32 and has_seg1.numel() == B, "has_seg1 must be int32 [B]")
    rope_dim = 0
    if inv_freq is not None:
        _cuda(inv_freq, "inv_freq")
        rope_dim = 2 * inv_freq.numel()
        _check(positions is not None and positions.is_cuda and positions.dtype == torch.int32
               and positions.numel() == B, "RoPE needs positions int32 [B]")
        inv_freq = inv_freq.float().contiguous()
    norm_weight = f32(norm_weight, (d,), "norm_weight")
    diag = None
    if page_pool is not None:
        for t, nm in ((page_table, "page_table"), (slot_pos, "slot_pos"), (page_pool, "page_pool")):
            _cuda(t, nm)
        _check(page_table.dtype == torch.int32 and slot_pos.dtype == torch.int32, "page tables must be int32")
        rb = d * bits // 8
        _check(page_pool.dtype == torch.uint8 and page_pool.dim() == 2 and page_pool.shape[1] == 64 * rb + 256,
               "page_pool must be uint8 [P, 64 * row_bytes + 256]")
        diag = rademacher_diag(d, seed, dev)
    out = torch.empty(B, d, dtype=torch.float32, device=dev) if want_out else None
    ptr = lambda t: None if t is None else t.data_ptr()
    # contiguous copies are held in locals until the launch is enqueued
    c0, z0 = c0.contiguous(), z0.contiguous()
    if c1 is not None:
        c1, z1 = c1.contiguous(), z1.contiguous()
    _lib.call("aether_compress_emit", c0.data_ptr(), z0.data_ptr(), ptr(bias0), m0, ptr(c1), ptr(z1),
              ptr(bias1 if c1 is not None else None), m1, ptr(has_seg1 if c1 is not None else None),
              _dt(c0, "c0"), B, d, ptr(positions), ptr(inv_freq), rope_dim, ptr(norm_weight), float(norm_eps),
              bits, ptr(diag), ptr(page_table), 0 if page_table is None else page_table.shape[1], ptr(slot_pos),
              0 if page_pool is None else page_pool.shape[0], ptr(page_pool), ptr(out), ptr(err), _stream(dev))
    return out


def tq_encode_lut(x: torch.Tensor, bits: int, seed: int = 42) -> Tuple[torch.Tensor, torch.Tensor]:
    """Lloyd-Max level format: (codes uint8 [..., D] or [..., D/2], scale fp32 [..., 1])."""
    from .codebook import device_codebook

    d = x.shape[-1]
    _cuda(x, "x")
    lead = x.shape[:-1]
    rows = x.numel() // d if d else 0
    lv, th = device_codebook(bits, x.device)
    codes = torch.empty(*lead, d if bits == 8 else d // 2, dtype=torch.uint8, device=x.device)
    scale = torch.empty(*lead, 1, dtype=torch.float32, device=x.device)
    _lib.call("aether_tq_encode_lut", x.data_ptr(), _dt(x, "x"), rows, d, bits,
              rademacher_diag(d, seed, x.device).data_ptr(), th.data_ptr(), float(lv[-1].item()), codes.data_ptr(),
              scale.data_ptr(), _stream(x.device))
    return codes, scale


def tq_decode_lut(codes: torch.Tensor, scale: torch.Tensor, bits: int, seed: int = 42,
                  out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    from .codebook import device_codebook

    _cuda(codes, "data")
    scale = scale.contiguous().float()
    d = codes.shape[-1] * (2 if bits == 4 else 1)
    rows = codes.numel() // codes.shape[-1] if codes.shape[-1] else 0
    _check(scale.numel() == rows, "scale must hold one value per vector")
    lv, _ = device_codebook(bits, codes.device)
    out = torch.empty(*codes.shape[:-1], d, dtype=out_dtype, device=codes.device)
    _lib.call("aether_tq_decode_lut", codes.data_ptr(), scale.data_ptr(), rows, d, bits,
              rademacher_diag(d, seed, codes.device).data_ptr(), lv.data_ptr(), out.data_ptr(), _dt(out, "out"),
              _stream(codes.device))
    return out


def tq_decode(codes: torch.Tensor, scale: torch.Tensor, bits: int, seed: int = 42,
              out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    _cuda(codes, "data")
    scale = scale.contiguous()
    _cuda(scale, "scale")
    d = codes.shape[-1] * (2 if bits == 4 else 1)
    rows = codes.numel() // codes.shape[-1] if codes.shape[-1] else 0
    _check(scale.numel() == rows, "scale must hold one value per vector")
    if scale.dtype != torch.float32:
        scale = scale.float()
    out = torch.empty(*codes.shape[:-1], d, dtype=out_dtype, device=codes.device)
    diag = rademacher_diag(d, seed, codes.device)
    _lib.call("aether_tq_decode", codes.data_ptr(), scale.data_ptr(), rows, d, bits, diag.data_ptr(),
              out.data_ptr(), _dt(out, "out"), _stream(codes.device))
    return out


def wht(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    _check(x.is_cuda, "x must be a CUDA tensor")
    xf = x.to(torch.float32).contiguous()
    out = torch.empty_like(xf)
    _lib.call("aether_wht", xf.data_ptr(), out.data_ptr(), xf.numel() // d if d else 0, d, _stream(x.device))
    return out


# ----------------------------------------------------------- reference ops
def sparse_sink_attention(q, kv, topk_indices, sink, softmax_scale: float) -> torch.Tensor:
    for t, nm in ((q, "q"), (kv, "kv"), (topk_indices, "topk_indices"), (sink, "sink")):
        _cuda(t, nm)
    _check(q.dim() == 4, "q must have shape [B, T, H, D]")
    _check(kv.dim() == 4, "kv must have shape [B, S, 2, D]")
    _check(kv.size(2) == 2, "kv third dimension must be 2 for [K, V]")
    _check(topk_indices.dim() == 3, "topk_indices must have shape [B, T, K]")
    _check(q.size(0) == kv.size(0), "q and kv batch dimensions must match")
    _check(q.size(0) == topk_indices.size(0), "q and topk_indices batch dimensions must match")
    _check(q.size(1) == topk_indices.size(1), "q and topk_indices target-token dimensions must match")
    _check(q.size(3) == kv.size(3), "q and kv head dimensions must match")
    _check(topk_indices.dtype in (torch.int64, torch.int32), "topk_indices must be int32 or int64")
    _check(sink.numel() == 1 or (sink.dim() == 1 and sink.size(0) == q.size(2)),
           "sink must be a scalar or a [num_heads] tensor")
    _check(kv.dtype == q.dtype and sink.dtype == q.dtype, "q, kv and sink must share a dtype")
    B, T, H, D = q.shape
    out = torch.empty_like(q)
    _lib.call("aether_sparse_sink_attention", q.data_ptr(), kv.data_ptr(), topk_indices.data_ptr(),
              int(topk_indices.dtype == torch.int64), sink.data_ptr(), sink.numel(), out.data_ptr(), _dt(q, "q"),
              B, T, H, D, kv.size(1), topk_indices.size(2), float(softmax_scale), _stream(q.device))
    return out


def tiled_prefill_attention(q, kv, sink, softmax_scale: float, tile_size: int = 256) -> torch.Tensor:
    for t, nm in ((q, "q"), (kv, "kv"), (sink, "sink")):
        _cuda(t, nm)
    _check(q.dim() == 4, "q must have shape [B, T, H, D]")
    _check(kv.dim() == 4, "kv must have shape [B, S, 2, D]")
    _check(kv.size(2) == 2, "kv third dimension must be 2 for [K, V]")
    _check(q.size(0) == kv.size(0), "q and kv batch dimensions must match")
    _check(q.size(3) == kv.size(3), "q and kv head dimensions must match")
    _check(tile_size > 0, "tile_size must be positive")
    _check(sink.numel() == 1 or (sink.dim() == 1 and sink.size(0) == q.size(2)),
           "sink must be a scalar or a [num_heads] tensor")
    _check(kv.dtype == q.dtype and sink.dtype == q.dtype, "q, kv and sink must share a dtype")
    B, T, H, D = q.shape
    out = torch.empty_like(q)
    _lib.call("aether_tiled_prefill_attention", q.data_ptr(), kv.data_ptr(), sink.data_ptr(), sink.numel(),
              out.data_ptr(), _dt(q, "q"), B, T, H, D, kv.size(1), float(softmax_scale), int(tile_size),
              _stream(q.device))
    return out


def csa_indexer_topk(index_q, index_kv, index_weight, k: int) -> torch.Tensor:
    for t, nm in ((index_q, "index_q"), (index_kv, "index_kv"), (index_weight, "index_weight")):
        _cuda(t, nm)
        _check(t.dtype == torch.float32, f"{nm} must be float32")
    _check(index_q.dim() == 3, "index_q must have shape [B, IH, IC]")
    _check(index_kv.dim() == 3, "index_kv must have shape [B, S, IC]")
    _check(index_weight.dim() == 2, "index_weight must have shape [B, IH]")
    _check(k > 0, "k must be positive")
    B, IH, IC = index_q.shape
    S = index_kv.size(1)
    out = torch.empty(B, k, dtype=torch.int64, device=index_q.device)
    scratch = torch.empty(max(B * S, 1), dtype=torch.float32, device=index_q.device)
    _lib.call("aether_csa_indexer_topk", index_q.data_ptr(), index_kv.data_ptr(), index_weight.data_ptr(), B, IH,
              IC, S, int(k), scratch.data_ptr(), out.data_ptr(), _stream(index_q.device))
    return out


def hca_compress(buffer_c, buffer_z) -> torch.Tensor:
    _cuda(buffer_c, "buffer_c")
    _cuda(buffer_z, "buffer_z")
    _check(buffer_c.dim() == 3, "buffer_c must have shape [B, M, D]")
    _check(buffer_z.dim() == 3, "buffer_z must have shape [B, M, D]")
    _check(buffer_c.shape == buffer_z.shape, "buffer_c and buffer_z must have the same shape")
    _check(buffer_c.dtype == buffer_z.dtype, "buffer_c and buffer_z must share a dtype")
    B, M, D = buffer_c.shape
    out = torch.empty(B, D, dtype=buffer_c.dtype, device=buffer_c.device)
    _lib.call("aether_hca_compress", buffer_c.data_ptr(), buffer_z.data_ptr(), out.data_ptr(),
              _dt(buffer_c, "buffer_c"), B, M, D, _stream(buffer_c.device))
    return out
