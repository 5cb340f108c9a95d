"""Paged TurboQuant KV cache and the fused decode entry points.

Cache layout in HBM (one ``TurboQuantPagedCache`` per attention layer):

    idx_pages [P, 64*R_i + 256] uint8   CSA indexer keys: 64 code rows of
                                        R_i = 64*bits/8 bytes, then 64 fp32 scales
    kv_pages  [P, 64*R_m + 256] uint8   shared K=V entries: 64 rows of
                                        R_m = 128*bits/8 bytes, then 64 scales

A page (codes and scales) is one contiguous block so one bulk (TMA) copy
moves it; ``idx_codes`` / ``idx_scale`` / ``kv_codes`` / ``kv_scale`` are
views into the pages.

Entry ``i`` of a sequence lives in physical page ``page_table[seq, i // 64]``
at slot ``i % 64``; the indexer and main streams share page ids.  Codes are
PolarQuant codes (aether_2b/turbo_quant.py:127-166): int8 for 8-bit, packed
signed nibbles (even element in the low nibble) for 4-bit.

This replaces the reference's LRU pool of de-quantized 128-token pages that
are gathered with ``torch.cat`` (aether_kernels/paged_kv_allocator.py:46-252,
aether_2b/serving.py:378-410, 486-493): pages stay quantized and the kernels
read them in place through the page table.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .ops import _check, _cuda, _stream, compress_emit, rademacher_diag, tq_encode_into_pages

PAGE = 64
HEAD_DIM = 128
INDEX_DIM = 64
INDEX_HEADS = 4


def _check_codebook(codebook: str) -> str:
    if codebook not in ("uniform", "lloyd-max"):
        raise ValueError(f"codebook must be 'uniform' or 'lloyd-max', got {codebook!r}")
    return codebook


class TurboQuantPagedCache:
    """Device page pool for one CSA or HCA layer (free-list page allocator).

    ``codebook`` selects the code format of the pages: "uniform" (the
    reference's PolarQuant levels) or "lloyd-max" (level indices into the
    Lloyd-Max N(0, 1) table, ``PolarQuant(bits, codebook="lloyd-max")``); the
    decode kernels apply the level table themselves."""

    def __init__(self, num_pages: int, bits: int, device, with_index: bool = True, seed: int = 42,
                 codebook: str = "uniform"):
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self.bits = bits
        self.seed = seed
        self.codebook = _check_codebook(codebook)
        self.num_pages = int(num_pages)
        self.device = torch.device(device)
        self.kv_row = HEAD_DIM * bits // 8
        self.idx_row = INDEX_DIM * bits // 8
        self.kv_pages = torch.zeros(num_pages, PAGE * self.kv_row + PAGE * 4, dtype=torch.uint8, device=self.device)
        self.idx_pages = (torch.zeros(num_pages, PAGE * self.idx_row + PAGE * 4, dtype=torch.uint8,
                                      device=self.device) if with_index else None)
        self._free: List[int] = list(range(num_pages - 1, -1, -1))

    @classmethod
    def from_pools(cls, kv_pages: torch.Tensor, idx_pages: Optional[torch.Tensor], bits: int,
                   seed: int = 42, codebook: str = "uniform") -> "TurboQuantPagedCache":
        """Wrap existing page pools (e.g. ``PagedKVAllocator.pool('kv')``) without
        copying; page allocation then belongs to whoever owns the pools."""
        if bits not in (4, 8):
            raise ValueError(f"bits must be 4 or 8, got {bits}")
        self = cls.__new__(cls)
        self.bits, self.seed, self.codebook = bits, seed, _check_codebook(codebook)
        self.kv_row, self.idx_row = HEAD_DIM * bits // 8, INDEX_DIM * bits // 8
        _check(kv_pages.dtype == torch.uint8 and kv_pages.dim() == 2
               and kv_pages.shape[1] == PAGE * self.kv_row + PAGE * 4, "kv_pages must be uint8 [P, page_bytes]")
        if idx_pages is not None:
            _check(idx_pages.dtype == torch.uint8 and idx_pages.shape == (kv_pages.shape[0], PAGE * self.idx_row + PAGE * 4),
                   "idx_pages must be uint8 [P, page_bytes] with kv_pages' page count")
        self.kv_pages, self.idx_pages = kv_pages, idx_pages
        self.num_pages = kv_pages.shape[0]
        self.device = kv_pages.device
        self._free = []
        return self

    # ------------------------------------------------------------- views
    @staticmethod
    def _codes(pages, row):
        return None if pages is None else pages[:, : PAGE * row].view(pages.shape[0], PAGE, row)

    @staticmethod
    def _scales(pages, row):
        return None if pages is None else pages[:, PAGE * row:].view(torch.float32)

    @property
    def kv_codes(self):
        return self._codes(self.kv_pages, self.kv_row)

    @property
    def kv_scale(self):
        return self._scales(self.kv_pages, self.kv_row)

    @property
    def idx_codes(self):
        return self._codes(self.idx_pages, self.idx_row)

    @property
    def idx_scale(self):
        return self._scales(self.idx_pages, self.idx_row)

    def tensors(self):
        return [t for t in (self.idx_pages, self.kv_pages) if t is not None]

    # ---------------------------------------------------------- page mgmt
    @property
    def free_pages(self) -> int:
        return len(self._free)

    def alloc_pages(self, n: int, generator: Optional[torch.Generator] = None) -> List[int]:
        if n > len(self._free):
            raise MemoryError(f"TurboQuant page pool exhausted: need {n}, {len(self._free)} free")
        if generator is not None:
            perm = torch.randperm(len(self._free), generator=generator)[:n].tolist()
            picked = [self._free[i] for i in perm]
            chosen = set(picked)
            self._free = [p for p in self._free if p not in chosen]
            return picked
        return [self._free.pop() for _ in range(n)]

    def release_pages(self, pages: Sequence[int]) -> None:
        self._free.extend(int(p) for p in pages)

    # --------------------------------------------------------------- write
    def write(self, page_table: torch.Tensor, start_pos: torch.Tensor, kv: torch.Tensor,
              index: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None) -> None:
        """Quantize ``kv`` [B, n, 128] (and ``index`` [B, n, 64]) and store
        them at logical positions start_pos[b] .. start_pos[b]+n-1."""
        if self.codebook == "lloyd-max":
            self._write_levels(page_table, start_pos, kv, self.kv_pages, self.kv_row)
            if index is not None:
                _check(self.idx_pages is not None, "this cache has no indexer stream")
                self._write_levels(page_table, start_pos, index, self.idx_pages, self.idx_row)
            return
        tq_encode_into_pages(kv, self.bits, page_table, start_pos, self.kv_pages, self.seed, err)
        if index is not None:
            _check(self.idx_pages is not None, "this cache has no indexer stream")
            tq_encode_into_pages(index, self.bits, page_table, start_pos, self.idx_pages, self.seed, err)

    def _write_levels(self, page_table, start_pos, x, pool, row):
        """Lloyd-Max format: encode densely, then scatter the rows to their
        page slots (a cache build step, not the decode path)."""
        from .ops import tq_encode_lut

        _check(x.dim() == 3, "x must have shape [B, n, D]")
        B, n, _ = x.shape
        if n == 0:
            return
        codes, scale = tq_encode_lut(x.contiguous(), self.bits, self.seed)
        pos = start_pos.long().view(B, 1) + torch.arange(n, device=x.device).view(1, n)
        page = page_table.long().gather(1, pos // PAGE)
        slot = pos % PAGE
        self._codes(pool, row)[page, slot] = codes
        self._scales(pool, row)[page, slot] = scale.squeeze(-1)


    # ---------------------------------------------------- compress-on-emit
    def emit_hca(self, page_table: torch.Tensor, slot_pos: torch.Tensor, buffer_c: torch.Tensor,
                 buffer_z: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor,
                 norm_weight: torch.Tensor, norm_eps: float = 1e-6, err: Optional[torch.Tensor] = None) -> None:
        """Finish one HCA block per sequence (aether_2b/serving.py:495-505):
        buffer_c / buffer_z [B, 128, 128] (bias already in z), entry written
        at logical position slot_pos[b]; one kernel launch."""
        _check(self.codebook == "uniform", "compress-on-emit writes the uniform code format")
        compress_emit(buffer_c, buffer_z, positions=positions, inv_freq=inv_freq, norm_weight=norm_weight,
                      norm_eps=norm_eps, bits=self.bits, page_table=page_table, slot_pos=slot_pos,
                      page_pool=self.kv_pages, seed=self.seed, want_out=False, err=err)

    def emit_csa(self, page_table: torch.Tensor, slot_pos: torch.Tensor, main: Sequence[torch.Tensor],
                 index: Sequence[torch.Tensor], has_prev: torch.Tensor, positions: torch.Tensor,
                 inv_freq: torch.Tensor, norm_weight: torch.Tensor, norm_eps: float = 1e-6,
                 err: Optional[torch.Tensor] = None) -> None:
        """Finish one CSA block per sequence (aether_2b/serving.py:540-575).
        ``main`` / ``index`` = (a_c, a_z, bias_a, prev_b_c, prev_b_z, bias_b)
        with [B, 4, d] halves and [4, d] biases; has_prev int32 [B] (0 for a
        sequence's first block).  Main entries get RoPE at ``positions`` and
        RMSNorm, index entries neither; two kernel launches."""
        _check(self.idx_pages is not None, "this cache has no indexer stream")
        _check(self.codebook == "uniform", "compress-on-emit writes the uniform code format")
        a_c, a_z, ba, b_c, b_z, bb = main
        compress_emit(a_c, a_z, ba, b_c, b_z, bb, has_prev, positions=positions, inv_freq=inv_freq,
                      norm_weight=norm_weight, norm_eps=norm_eps, bits=self.bits, page_table=page_table,
                      slot_pos=slot_pos, page_pool=self.kv_pages, seed=self.seed, want_out=False, err=err)
        a_c, a_z, ba, b_c, b_z, bb = index
        compress_emit(a_c, a_z, ba, b_c, b_z, bb, has_prev, bits=self.bits, page_table=page_table,
                      slot_pos=slot_pos, page_pool=self.idx_pages, seed=self.seed, want_out=False, err=err)

def csa_workspace_bytes(batch: int, max_nblocks: int) -> int:
    """Workspace bytes of ``csa_decode_paged`` (u32 score key per visible block)."""
    return int(_lib.load().aether_csa_decode_workspace_bytes(int(batch), int(max_nblocks)))


def _opt_ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def csa_decode_paged(
    q: torch.Tensor,
    index_q: torch.Tensor,
    index_weight: torch.Tensor,
    sink: torch.Tensor,
    window: torch.Tensor,
    window_len: torch.Tensor,
    cache: TurboQuantPagedCache,
    page_table: torch.Tensor,
    nblocks: torch.Tensor,
    softmax_scale: float,
    top_k: int = 256,
    out: Optional[torch.Tensor] = None,
    indices: Optional[torch.Tensor] = None,
    err: Optional[torch.Tensor] = None,
    scores: Optional[torch.Tensor] = None,
    overlap_prefetch: bool = False,
    workspace: Optional[torch.Tensor] = None,
    rope_positions: Optional[torch.Tensor] = None,
    rope_inv_freq: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """One fused CSA decode step for a batch of sequences.

    q [B, H, 128] bf16 (post-RoPE, post-norm), index_q [B, 4, 64] fp32,
    index_weight [B, 4] fp32 raw head weights (softplus applied in-kernel),
    sink [H] fp32, window [B, W, 128] bf16 (oldest first, ``window_len[b]``
    valid rows), page_table [B, max_pages] int32, nblocks [B] int32 visible
    compressed blocks.  Returns ``(out [B, H, 128] bf16, indices [B, top_k]
    int32)``: the attention output before the inverse output RoPE (what
    ``AttentionKernelBackend.sparse_attention`` returns) and the selected
    block indices in ascending order, -1 padded.

    Two kernels run per step: a score kernel and a select/attend kernel with
    a 2-CTA cluster per sequence.  ``overlap_prefetch=True`` launches
    with programmatic dependent launch: the kernel may start while the
    previous kernel on the stream is still running and, before waiting for
    it, reads ``page_table``, ``nblocks``, ``window_len``, the cache pages and
    every window row except the newest.  Use it only when the immediately
    preceding kernel writes none of those.  ``scores`` (optional fp32
    [B, >= max_pages * 64]) receives every visible block's index score.
    ``workspace`` (optional uint8 tensor of ``csa_workspace_bytes(B, max_pages
    * 64)`` bytes) holds the per-block score keys between the two kernels;
    it is allocated per call when not given (contents need no clearing).
    ``rope_positions`` (int32 [B]) with ``rope_inv_freq`` (fp32 [rope_dim/2])
    fuse the inverse output RoPE of aether_2b/serving.py:469-472 into the
    store: the last rope_dim channels are rotated by -position.
    """
    B, H, D = q.shape
    _check(D == HEAD_DIM, f"head_dim must be {HEAD_DIM}")
    for t, nm in ((q, "q"), (index_q, "index_q"), (index_weight, "index_weight"), (sink, "sink"),
                  (window, "window"), (window_len, "window_len"), (page_table, "page_table"),
                  (nblocks, "nblocks")):
        _cuda(t, nm)
    _check(q.dtype == torch.bfloat16 and window.dtype == torch.bfloat16, "q and window must be bfloat16")
    _check(index_q.dtype == torch.float32 and index_weight.dtype == torch.float32 and sink.dtype == torch.float32,
           "index_q, index_weight and sink must be float32")
    _check(tuple(index_q.shape) == (B, INDEX_HEADS, INDEX_DIM), "index_q must have shape [B, 4, 64]")
    _check(page_table.dtype == torch.int32 and nblocks.dtype == torch.int32 and window_len.dtype == torch.int32,
           "page_table, nblocks and window_len must be int32")
    _check(cache.idx_pages is not None, "CSA decode needs a cache with an indexer stream")
    dev = q.device
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
    if indices is None:
        indices = torch.empty(B, top_k, dtype=torch.int32, device=dev)
    common = (
        q.data_ptr(), index_q.data_ptr(), index_weight.data_ptr(), sink.data_ptr(), window.data_ptr(),
        window_len.data_ptr(), cache.idx_pages.data_ptr(), cache.kv_pages.data_ptr(), page_table.data_ptr(), page_table.shape[1], cache.num_pages,
        nblocks.data_ptr(), page_table.shape[1] * PAGE,
        rademacher_diag(INDEX_DIM, cache.seed, dev).data_ptr(), rademacher_diag(HEAD_DIM, cache.seed, dev).data_ptr(),
        B, H, window.shape[1], cache.bits, int(top_k), float(softmax_scale),
        out.data_ptr(), indices.data_ptr(),
    )
    need = csa_workspace_bytes(B, page_table.shape[1] * PAGE)
    if workspace is None:
        workspace = torch.zeros(max(need, 16), dtype=torch.uint8, device=dev)
    _check(workspace.is_cuda and workspace.numel() * workspace.element_size() >= need,
           f"workspace must hold {need} bytes")
    if getattr(cache, "codebook", "uniform") == "lloyd-max":
        from .codebook import device_codebook

        _check(scores is None and rope_inv_freq is None,
               "a Lloyd-Max cache decodes without score output or fused output RoPE")
        lv, _ = device_codebook(cache.bits, dev)
        _lib.call("aether_csa_decode_paged_levels", *common[:21], lv.data_ptr(), *common[21:], workspace.data_ptr(),
                  _opt_ptr(err), int(overlap_prefetch), _stream(dev))
        return out, indices
    if rope_inv_freq is not None:
        _check(scores is None, "the fused output RoPE does not write scores")
        _cuda(rope_positions, "rope_positions")
        _cuda(rope_inv_freq, "rope_inv_freq")
        _check(rope_positions.dtype == torch.int32 and rope_positions.numel() == B, "rope_positions must be int32 [B]")
        _check(rope_inv_freq.dtype == torch.float32, "rope_inv_freq must be float32")
        _lib.call("aether_csa_decode_paged_rope", *common, workspace.data_ptr(), _opt_ptr(err),
                  int(overlap_prefetch), rope_positions.data_ptr(), rope_inv_freq.data_ptr(),
                  2 * rope_inv_freq.numel(), _stream(dev))
    elif scores is None:
        _lib.call("aether_csa_decode_paged", *common, workspace.data_ptr(), _opt_ptr(err), 0,
                  int(overlap_prefetch), _stream(dev))
    else:
        _cuda(scores, "scores")
        _check(scores.dtype == torch.float32 and scores.shape[0] == B and scores.shape[1] >= page_table.shape[1] * PAGE,
               "scores must be float32 [B, >= max_pages * 64]")
        _lib.call("aether_csa_decode_paged_scores", *common, scores.data_ptr(), scores.shape[1],
                  workspace.data_ptr(), _opt_ptr(err), 0, int(overlap_prefetch), _stream(dev))
    return out, indices



class HostDecodeBuffers:
    """Device staging for ``csa_decode_paged_host``: the step inputs packed as
    [q | index_q | index_weight | window_len | nblocks] and the results as
    [out | indices], each field 256-byte aligned."""

    FIELDS = ("q", "index_q", "index_weight", "window_len", "nblocks")

    def __init__(self, batch: int, heads: int = 12, top_k: int = 256, device="cuda"):
        self.batch, self.heads, self.top_k = batch, heads, top_k
        self.device = torch.device(device)
        self.in_shapes = [((batch, heads, HEAD_DIM), torch.bfloat16), ((batch, INDEX_HEADS, INDEX_DIM), torch.float32),
                          ((batch, INDEX_HEADS), torch.float32), ((batch,), torch.int32), ((batch,), torch.int32)]
        self.out_shapes = [((batch, heads, HEAD_DIM), torch.bfloat16), ((batch, top_k), torch.int32)]
        self.in_offsets, self.in_bytes = self._layout(self.in_shapes)
        self.out_offsets, self.out_bytes = self._layout(self.out_shapes)
        self.dev_in = torch.empty(self.in_bytes, dtype=torch.uint8, device=self.device)
        self.dev_out = torch.empty(self.out_bytes, dtype=torch.uint8, device=self.device)
        self.inputs = self._views(self.dev_in, self.in_shapes, self.in_offsets)
        self.out, self.indices = self._views(self.dev_out, self.out_shapes, self.out_offsets)
        self._ws_key, self._ws_need, self._diags = None, 0, (0, 0)
        # copy-completion words [input copied, output copied] and the step
        # sequence number written into them (steps with copy streams)
        self.slot_flags = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.seq = 0

    @staticmethod
    def _layout(shapes):
        offs, off = [], 0
        for shape, dt in shapes:
            offs.append(off)
            n = 1
            for d in shape:
                n *= d
            off += (n * torch.empty((), dtype=dt).element_size() + 255) // 256 * 256
        return offs, off

    @staticmethod
    def _views(buf, shapes, offs):
        out = []
        for (shape, dt), o in zip(shapes, offs):
            n = 1
            for d in shape:
                n *= d
            es = torch.empty((), dtype=dt).element_size()
            out.append(buf[o: o + n * es].view(dt).view(shape))
        return out

    def pack_inputs(self, q, index_q, index_weight, window_len, nblocks) -> torch.Tensor:
        """Pinned host buffer holding one step's inputs in the packed layout."""
        host = torch.empty(self.in_bytes, dtype=torch.uint8).pin_memory()
        for t, (shape, dt), o in zip((q, index_q, index_weight, window_len, nblocks), self.in_shapes, self.in_offsets):
            _check(tuple(t.shape) == shape and t.dtype == dt, f"input must be {dt} {list(shape)}")
            b = t.detach().contiguous().cpu().view(torch.uint8).view(-1)
            host[o: o + b.numel()].copy_(b)
        return host

    def new_host_output(self) -> torch.Tensor:
        return torch.empty(self.out_bytes, dtype=torch.uint8).pin_memory()

    def unpack_outputs(self, host_out: torch.Tensor):
        """(out [B, H, 128] bf16, indices [B, top_k] int32) views of a host result buffer."""
        return tuple(self._views(host_out, self.out_shapes, self.out_offsets))


class CopyStreams:
    """Copy streams and per-slot events for overlapped ``csa_decode_paged_host``
    calls: a step's input copy runs on ``h2d``, its output copy on ``d2h``;
    callers alternate two staging slots (``HostDecodeBuffers``)."""

    def __init__(self, device, slots: int = 2):
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.events = [tuple(torch.cuda.Event() for _ in range(3)) for _ in range(slots)]
        # torch creates an event's CUDA handle on its first record
        for evs in self.events:
            for e in evs:
                e.record(self.h2d)
        self.h2d.synchronize()

    def last_output(self, slot: int) -> torch.cuda.Event:
        """Event recorded after the slot's latest output copy."""
        return self.events[slot][2]


def csa_decode_paged_host(bufs: HostDecodeBuffers, host_in: torch.Tensor, host_out: torch.Tensor,
                          sink: torch.Tensor, window: torch.Tensor, cache: TurboQuantPagedCache,
                          page_table: torch.Tensor, softmax_scale: float, workspace: torch.Tensor,
                          err: Optional[torch.Tensor] = None, copies: Optional[CopyStreams] = None,
                          slot: int = 0, overlap_prefetch: bool = False) -> None:
    """One CSA decode step with host buffers, enqueued by a single C call: the
    packed inputs are copied from pinned ``host_in`` to the device, the decode
    runs on the current stream, and the packed output and indices are copied
    to pinned ``host_out`` (read them with ``bufs.unpack_outputs`` once the
    copy has completed).  With ``copies`` the transfers run on its streams,
    ordered by the slot's events and by ``bufs``' copy-completion words, which
    the kernels poll; pass a different ``bufs`` per slot, and the same slot
    index with the same ``bufs`` every time.  ``overlap_prefetch`` as in
    ``csa_decode_paged``: only when no kernel before this step on the stream
    writes the cache pages or the page table."""
    # host buffers from pack_inputs / new_host_output are pinned; others work
    # but their copies are synchronous
    _check(host_in.numel() >= bufs.in_bytes and host_out.numel() >= bufs.out_bytes, "host buffers too small")
    _check(cache.idx_pages is not None, "CSA decode needs a cache with an indexer stream")
    q, iq, iw, wl, nb = bufs.inputs
    dev = bufs.device
    key = (page_table.shape[1], cache.seed)
    if bufs._ws_key != key:  # per-shape constants, computed once
        bufs._ws_need = csa_workspace_bytes(bufs.batch, page_table.shape[1] * PAGE)
        bufs._diags = (rademacher_diag(INDEX_DIM, cache.seed, dev).data_ptr(),
                       rademacher_diag(HEAD_DIM, cache.seed, dev).data_ptr())
        bufs._ws_key = key
    _check(workspace.is_cuda and workspace.numel() * workspace.element_size() >= bufs._ws_need,
           f"workspace must hold {bufs._ws_need} bytes")
    if copies is not None:
        bufs.seq = (bufs.seq + 1) & 0xFFFFFFFF
    _lib.call("aether_csa_decode_paged_host", host_in.data_ptr(), bufs.dev_in.data_ptr(), bufs.in_bytes,
              host_out.data_ptr(), bufs.dev_out.data_ptr(), bufs.out_bytes, q.data_ptr(), iq.data_ptr(),
              iw.data_ptr(), sink.data_ptr(), window.data_ptr(), wl.data_ptr(), cache.idx_pages.data_ptr(),
              cache.kv_pages.data_ptr(), page_table.data_ptr(), page_table.shape[1], cache.num_pages, nb.data_ptr(),
              page_table.shape[1] * PAGE, bufs._diags[0], bufs._diags[1], bufs.batch, bufs.heads, window.shape[1],
              cache.bits, bufs.top_k, float(softmax_scale), bufs.out.data_ptr(), bufs.indices.data_ptr(),
              workspace.data_ptr(), _opt_ptr(err), int(overlap_prefetch), _stream(dev),
              *((copies.h2d.cuda_stream, copies.d2h.cuda_stream, *[e.cuda_event for e in copies.events[slot]],
                 bufs.slot_flags.data_ptr(), bufs.seq) if copies is not None else (None,) * 6 + (0,)))

class CsaDecodeHostPlan:
    """A prepared host-buffer CSA decode (``aether_csa_decode_host_plan_*``):
    two staging slots, copy streams, the cache and the launch shape are bound
    once; each ``step`` enqueues one step's input copy from pinned host
    memory, the decode and the output copy to pinned host memory with one
    short C call, alternating the staging slots so a step's copies overlap its
    neighbours' kernels.  Same results as ``csa_decode_paged_host``.
    ``max_pages`` is the widest page table a step may pass.

    ``overlap_prefetch`` as in ``csa_decode_paged``: only when no kernel
    before a step on the stream writes the cache pages or the page table."""

    def __init__(self, cache: TurboQuantPagedCache, batch: int, max_pages: int, heads: int = 12,
                 top_k: int = 256, window: int = 128, err: Optional[torch.Tensor] = None,
                 overlap_prefetch: bool = False, device="cuda"):
        import ctypes
        _check(cache.idx_pages is not None, "CSA decode needs a cache with an indexer stream")
        self.device = torch.device(device)
        self.slots = [HostDecodeBuffers(batch, heads, top_k, self.device) for _ in range(2)]
        self.in_bytes, self.out_bytes = self.slots[0].in_bytes, self.slots[0].out_bytes
        self.table_stride, self.window = max_pages, window
        self._flags = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._ws = torch.zeros(csa_workspace_bytes(batch, max_pages * PAGE), dtype=torch.uint8, device=self.device)
        self._diags = (rademacher_diag(INDEX_DIM, cache.seed, self.device),
                       rademacher_diag(HEAD_DIM, cache.seed, self.device))
        self._cache, self._err = cache, err
        in_off = (ctypes.c_size_t * 5)(*self.slots[0].in_offsets)
        out_off = (ctypes.c_size_t * 2)(*self.slots[0].out_offsets)
        handle = ctypes.c_void_p()
        a, b = self.slots
        _lib.call("aether_csa_decode_host_plan_create", a.dev_in.data_ptr(), b.dev_in.data_ptr(), self.in_bytes,
                  in_off, a.dev_out.data_ptr(), b.dev_out.data_ptr(), self.out_bytes, out_off,
                  self._flags.data_ptr(), cache.idx_pages.data_ptr(), cache.kv_pages.data_ptr(), max_pages,
                  cache.num_pages, max_pages * PAGE, self._diags[0].data_ptr(), self._diags[1].data_ptr(), batch,
                  heads, window, cache.bits, top_k, self._ws.data_ptr(),
                  _opt_ptr(err), int(overlap_prefetch), ctypes.byref(handle))
        self._h = handle.value
        lib = _lib.load()
        self._step, self._fence, self._destroy = (lib.aether_csa_decode_host_plan_step,
                                                  lib.aether_csa_decode_host_plan_fence,
                                                  lib.aether_csa_decode_host_plan_destroy)

    def pack_inputs(self, q, index_q, index_weight, window_len, nblocks) -> torch.Tensor:
        """Pinned host buffer holding one step's inputs in the packed layout."""
        return self.slots[0].pack_inputs(q, index_q, index_weight, window_len, nblocks)

    def new_host_output(self) -> torch.Tensor:
        return self.slots[0].new_host_output()

    def unpack_outputs(self, host_out: torch.Tensor):
        """(out [B, H, 128] bf16, indices [B, top_k] int32) views of a host result buffer."""
        return self.slots[0].unpack_outputs(host_out)

    def step(self, host_in: torch.Tensor, host_out: torch.Tensor, page_table: torch.Tensor, sink: torch.Tensor,
             window: torch.Tensor, softmax_scale: float) -> None:
        """Enqueue one step on the current stream: pinned ``host_in`` (from
        ``pack_inputs``) in, results to pinned ``host_out`` once the plan's
        copies are done (``fence(wait_for_copies=True)`` then synchronise)."""
        _check(self._h is not None, "plan is closed")
        _check(window.shape[:2] == (self.slots[0].batch, self.window), "window shape differs from the plan")
        rc = self._step(self._h, host_in.data_ptr(), host_out.data_ptr(), page_table.data_ptr(), page_table.shape[1],
                        sink.data_ptr(), window.data_ptr(), softmax_scale, _stream(self.device))
        if rc != 0:
            raise _lib.AetherKernelError(f"aether_csa_decode_host_plan_step failed ({rc}): {_lib.last_error()}")

    def fence(self, wait_for_copies: bool) -> None:
        """Order the plan's copy streams against the current stream (see the C entry)."""
        _lib.call("aether_csa_decode_host_plan_fence", self._h, _stream(self.device), int(wait_for_copies))

    def close(self) -> None:
        if self._h is not None:
            self._destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def hca_decode_paged(
    q: torch.Tensor,
    sink: torch.Tensor,
    window: torch.Tensor,
    window_len: torch.Tensor,
    cache: TurboQuantPagedCache,
    page_table: torch.Tensor,
    nblocks: torch.Tensor,
    softmax_scale: float,
    out: Optional[torch.Tensor] = None,
    err: Optional[torch.Tensor] = None,
    overlap_prefetch: bool = False,
) -> torch.Tensor:
    """One fused HCA decode step: attention over every visible compressed
    block plus the sliding window (aether_2b/serving.py:507-522).

    One 4-CTA cluster per sequence.  ``overlap_prefetch=True`` launches with programmatic dependent launch: before waiting for the
    previous kernel on the stream the kernel reads ``page_table``,
    ``nblocks``, ``window_len``, the cache pages and every window row except
    the newest; use it only when that kernel writes none of those."""
    B, H, D = q.shape
    _check(D == HEAD_DIM, f"head_dim must be {HEAD_DIM}")
    for t, nm in ((q, "q"), (sink, "sink"), (window, "window"), (window_len, "window_len"),
                  (page_table, "page_table"), (nblocks, "nblocks")):
        _cuda(t, nm)
    _check(q.dtype == torch.bfloat16 and window.dtype == torch.bfloat16, "q and window must be bfloat16")
    _check(sink.dtype == torch.float32, "sink must be float32")
    dev = q.device
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
    head = (q.data_ptr(), sink.data_ptr(), window.data_ptr(), window_len.data_ptr(), cache.kv_pages.data_ptr(),
            page_table.data_ptr(), page_table.shape[1], cache.num_pages, nblocks.data_ptr(),
            page_table.shape[1] * PAGE, rademacher_diag(HEAD_DIM, cache.seed, dev).data_ptr(),
            B, H, window.shape[1], cache.bits, float(softmax_scale))
    if getattr(cache, "codebook", "uniform") == "lloyd-max":
        from .codebook import device_codebook

        lv, _ = device_codebook(cache.bits, dev)
        _lib.call("aether_hca_decode_paged_levels", *head, lv.data_ptr(), out.data_ptr(), _opt_ptr(err),
                  int(overlap_prefetch), _stream(dev))
        return out
    _lib.call("aether_hca_decode_paged", *head, out.data_ptr(), _opt_ptr(err), 0, int(overlap_prefetch), _stream(dev))
    return out
