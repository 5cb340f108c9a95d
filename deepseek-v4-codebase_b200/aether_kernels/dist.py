"""Multi-device CSA decode.

Two layouts (new design: the reference serves one sequence per process and
only shards layers, aether_2b/serving.py:1053-1076):

* request partitioning -- each rank decodes its own sequences with
  ``csa_decode_paged``; no collective on the data path.
* context partitioning (``csa_decode_context_parallel``) -- one long
  sequence's compressed blocks are split into contiguous ranges, one per
  rank.  Each rank keeps the exact top-k of every 8192-block chunk of its
  range; the candidate lists are all-gathered (NCCL over NVLink) and every
  rank takes the exact global top-k of the union (a global winner is always
  in its own chunk's top-k; ties go to the lower block id on every rank);
  each rank attends to the winners it holds (the last rank also to the
  window) and the partial results (O, max, sum) are all-gathered and merged
  by log-sum-exp with the sink counted once.

The collective orchestration (``context_parallel_step``) takes the three
compute steps as callables, so the same code runs with the CUDA kernels over
NCCL and, in the CPU tests, with reference-math callables over gloo.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib
from .ops import _check, _cuda, _stream, rademacher_diag
from .paged import HEAD_DIM, INDEX_DIM, PAGE, TurboQuantPagedCache, csa_workspace_bytes

CHUNK = 8192


def chunks_for(max_nblocks: int) -> int:
    return max(1, (max_nblocks + CHUNK - 1) // CHUNK)


# ------------------------------------------------------------ device steps
def local_candidates(index_q, index_weight, cache: TurboQuantPagedCache, page_table, nblocks, id_base: int,
                     top_k: int = 256, err: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Exact top_k of every 8192-block chunk of this device's blocks.

    Returns (keys, ids), each int32 [B, chunks * top_k]; keys are the
    order-preserving u32 score keys (bit patterns, 0 = padding), ids the
    global block ids (ascending, -1 = padding)."""
    B = index_q.shape[0]
    max_nb = page_table.shape[1] * PAGE
    ch = chunks_for(max_nb)
    dev = index_q.device
    keys = torch.empty(B, ch * top_k, dtype=torch.int32, device=dev)
    ids = torch.empty(B, ch * top_k, dtype=torch.int32, device=dev)
    ws = torch.empty(max(csa_workspace_bytes(B, max_nb), 16), dtype=torch.uint8, device=dev)
    _lib.call("aether_csa_local_candidates", index_q.data_ptr(), index_weight.data_ptr(), cache.idx_pages.data_ptr(),
              page_table.data_ptr(), page_table.shape[1], cache.num_pages, nblocks.data_ptr(), max_nb,
              rademacher_diag(INDEX_DIM, cache.seed, dev).data_ptr(), B, cache.bits, int(top_k), int(id_base),
              keys.data_ptr(), ids.data_ptr(), ws.data_ptr(), None if err is None else err.data_ptr(), _stream(dev))
    return keys, ids


def attend_candidates(q, sink, window, window_len, cache: TurboQuantPagedCache, page_table, nblocks, cand_keys,
                      cand_ids, id_base: int, softmax_scale: float, top_k: int = 256, partial: bool = True,
                      err: Optional[torch.Tensor] = None):
    """Exact top_k of the merged candidates, attention over the winners held
    here.  partial=True returns (part_o fp32 [B,H,128], part_ml fp32
    [B,H,2], selected int32 [B,top_k]); otherwise (out bf16 [B,H,128], selected)."""
    B, H, D = q.shape
    _check(D == HEAD_DIM, f"head_dim must be {HEAD_DIM}")
    dev = q.device
    for t, nm in ((cand_keys, "cand_keys"), (cand_ids, "cand_ids")):
        _cuda(t, nm)
    n = cand_keys.shape[1]
    sel = torch.empty(B, top_k, dtype=torch.int32, device=dev)
    if partial:
        # O and (max, sum) adjacent in one buffer: one collective moves both
        flat = torch.empty(B * H * (D + 2), dtype=torch.float32, device=dev)
        po = flat[: B * H * D].view(B, H, D)
        pml = flat[B * H * D:].view(B, H, 2)
        out_ptr, po_ptr, pml_ptr = None, po.data_ptr(), pml.data_ptr()
    else:
        out = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
        out_ptr, po_ptr, pml_ptr = out.data_ptr(), None, None
    _lib.call("aether_csa_attend_candidates", q.data_ptr(), sink.data_ptr(), window.data_ptr(), window_len.data_ptr(),
              cache.kv_pages.data_ptr(), page_table.data_ptr(), page_table.shape[1], cache.num_pages,
              nblocks.data_ptr(), page_table.shape[1] * PAGE, rademacher_diag(HEAD_DIM, cache.seed, dev).data_ptr(),
              cand_keys.data_ptr(), cand_ids.data_ptr(), n, n, int(id_base), B, H, window.shape[1], cache.bits,
              int(top_k), float(softmax_scale), out_ptr, sel.data_ptr(), po_ptr, pml_ptr,
              None if err is None else err.data_ptr(), _stream(dev))
    return (po, pml, sel) if partial else (out, sel)


def lse_merge(part_o: torch.Tensor, part_ml: torch.Tensor, sink: torch.Tensor) -> torch.Tensor:
    """part_o [G,B,H,128] fp32, part_ml [G,B,H,2] fp32, sink [H] fp32 -> bf16 [B,H,128].
    Each rank's block must be contiguous; the rank dimension may be strided
    (rows of an all-gathered packed buffer)."""
    G, B, H, D = part_o.shape
    out = torch.empty(B, H, D, dtype=torch.bfloat16, device=part_o.device)
    if not (part_o[0].is_contiguous() and part_ml[0].is_contiguous()):
        part_o, part_ml = part_o.contiguous(), part_ml.contiguous()  # kept alive past the launch
    _lib.call("aether_lse_merge_strided", part_o.data_ptr(), part_ml.data_ptr(), part_o.stride(0),
              part_ml.stride(0), sink.data_ptr(), G, B, H, out.data_ptr(), _stream(part_o.device))
    return out


# ---------------------------------------------------------- orchestration
def context_parallel_step(candidates_fn: Callable[[], Tuple[torch.Tensor, torch.Tensor]],
                          attend_fn: Callable[[torch.Tensor, torch.Tensor], Tuple[torch.Tensor, torch.Tensor,
                                                                                  torch.Tensor]],
                          merge_fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor],
                          group=None):
    """One context-parallel decode step.  candidates_fn() -> (keys, ids) of
    this rank; attend_fn(all_keys, all_ids) -> (part_o, part_ml, selected);
    merge_fn(stacked part_o, stacked part_ml) -> output.  Candidate lists are
    concatenated in rank order, so ids stay ascending when rank r holds the
    r-th contiguous block range."""
    world = dist.get_world_size(group)
    keys, ids = candidates_fn()

    def gather_rows(t):  # per rank t -> [world, *t.shape] (flat buffers: every backend accepts them)
        g = torch.empty(world * t.numel(), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(g, t.contiguous().view(-1), group=group)
        return g.view((world,) + tuple(t.shape))

    if keys.dtype == ids.dtype and keys.shape == ids.shape:  # one collective for both
        g = gather_rows(torch.stack([keys, ids]))             # [world, 2, B, n]
        gk, gi = g[:, 0], g[:, 1]
    else:
        gk, gi = gather_rows(keys), gather_rows(ids)
    B = keys.shape[0]
    all_keys = gk.transpose(0, 1).reshape(B, -1).contiguous()
    all_ids = gi.transpose(0, 1).reshape(B, -1).contiguous()
    po, pml, sel = attend_fn(all_keys, all_ids)
    npo = po.numel()
    adjacent = (po.is_contiguous() and pml.is_contiguous() and po.dtype == pml.dtype
                and pml.data_ptr() == po.data_ptr() + npo * po.element_size())
    flat = torch.as_strided(po, (npo + pml.numel(),), (1,)) if adjacent else \
        torch.cat([po.reshape(-1), pml.reshape(-1)])
    gp = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(gp, flat, group=group)
    gp = gp.view(world, flat.numel())
    return merge_fn(gp[:, :npo].view(world, *po.shape), gp[:, npo:].view(world, *pml.shape)), sel


def csa_decode_context_parallel(q, index_q, index_weight, sink, window, window_len, cache: TurboQuantPagedCache,
                                page_table, nblocks, id_base: int, softmax_scale: float, top_k: int = 256,
                                group=None, err: Optional[torch.Tensor] = None):
    """CSA decode for sequences whose blocks are split across the ranks of
    ``group``: this rank holds global blocks [id_base, id_base + nblocks[b]).
    ``window_len`` is 0 on every rank but the one holding the window.
    Returns (out bf16 [B,H,128], selected global block ids [B,top_k])."""
    return context_parallel_step(
        lambda: local_candidates(index_q, index_weight, cache, page_table, nblocks, id_base, top_k, err),
        lambda k, i: attend_candidates(q, sink, window, window_len, cache, page_table, nblocks, k, i, id_base,
                                       softmax_scale, top_k, partial=True, err=err),
        lambda po, pml: lse_merge(po, pml, sink),
        group=group)


# ------------------------------------------------------ peer-memory exchange
def _pad16(n: int) -> int:
    return (n + 15) & ~15


def peer_layout(batch: int, heads: int, n: int, world: int, control_bytes: int = 256) -> dict:
    """Byte layout of one rank's exchange buffer: control area; candidate
    keys [batch][world * n] int32 (rank r's list at column r * n); candidate
    ids, the same shape right after the keys (so keys and ids of a rank are
    2 * batch rows of one strided copy); then ``world`` partial slots, each O
    [batch][heads][128] fp32 followed by (max, sum) [batch][heads][2] fp32
    and padded to 16 bytes."""
    row = world * n * 4
    off_k = control_bytes
    off_i = off_k + batch * row
    off_p = _pad16(off_i + batch * row)
    o_bytes = batch * heads * HEAD_DIM * 4
    slot = _pad16(o_bytes + batch * heads * 2 * 4)
    return dict(row_bytes=row, off_k=off_k, off_i=off_i, off_p=off_p, o_bytes=o_bytes, slot=slot,
                total=off_p + world * slot)


class PeerContextParallel:
    """Context-parallel CSA decode whose two exchanges are stores into the
    other GPUs' memory (``aether_peer_push`` / ``aether_peer_wait``) instead
    of NCCL all-gathers: the same math as ``csa_decode_context_parallel``
    (candidate lists in rank order, exact global top-k on every rank, the
    log-sum-exp merge with the sink counted once), with no collective launch
    and no host synchronisation inside a step, so a step can be captured in a
    CUDA graph.

    Every rank builds the plan with the same batch, head count and local
    block capacity; the constructor exchanges CUDA IPC handles over
    ``group`` (any backend).  Layout of each rank's exchange buffer: control
    area, candidate keys [B][G * n], candidate ids [B][G * n] (rank r's
    lists at column r * n), then G partial slots (O [B][H][128] and (max,
    sum) [B][H][2], fp32).  Call ``close()`` on every rank when done."""

    def __init__(self, batch: int, heads: int, max_local_blocks: int, top_k: int = 256, group=None, device=None):
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        self.B, self.H, self.top_k = batch, heads, top_k
        self.dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.max_nb = (max(max_local_blocks, 1) + PAGE - 1) // PAGE * PAGE
        self.n = chunks_for(self.max_nb) * top_k
        lib = _lib.load()
        lay = peer_layout(batch, heads, self.n, self.G, int(lib.aether_cp_control_bytes()))
        self.off_k, self.off_i, self.off_p = lay["off_k"], lay["off_i"], lay["off_p"]
        self.o_bytes, self.slot, total = lay["o_bytes"], lay["slot"], lay["total"]
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        _lib.call("aether_cp_buffer_create", total, ctypes.byref(ptr), handle)
        self._own = ptr.value
        handles = [None] * self.G
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened, bases = [], []
        for g, h in enumerate(handles):
            if g == self.rank:
                bases.append(self._own)
                continue
            peer = ctypes.c_void_p()
            _lib.call("aether_cp_buffer_open", ctypes.create_string_buffer(h, 64), ctypes.byref(peer))
            self._opened.append(peer.value)
            bases.append(peer.value)
        self._bases = (ctypes.c_void_p * self.G)(*bases)
        # local staging, allocated once (a captured step allocates nothing)
        self.cand = torch.empty(2, batch, self.n, dtype=torch.int32, device=self.dev)
        self.part = torch.empty(self.slot // 4, dtype=torch.float32, device=self.dev)
        self.ws = torch.empty(max(csa_workspace_bytes(batch, self.max_nb), 16), dtype=torch.uint8, device=self.dev)
        self.sel = torch.empty(batch, top_k, dtype=torch.int32, device=self.dev)
        self.out = torch.empty(batch, heads, HEAD_DIM, dtype=torch.bfloat16, device=self.dev)
        dist.barrier(group=group)

    def step(self, q, index_q, index_weight, sink, window, window_len, cache: TurboQuantPagedCache, page_table,
             nblocks, id_base: int, softmax_scale: float, err: Optional[torch.Tensor] = None):
        """One decode step (same arguments as csa_decode_context_parallel);
        returns (out bf16 [B,H,128], selected global block ids [B,top_k]),
        both buffers of the plan, overwritten by the next step."""
        B, H, n, G = self.B, self.H, self.n, self.G
        _check(tuple(q.shape) == (B, H, HEAD_DIM), f"q must be [{B}, {H}, {HEAD_DIM}]")
        _check(page_table.shape[1] * PAGE <= self.max_nb, "page table exceeds the plan's local block capacity")
        dev = q.device
        st = _stream(dev)
        ep = None if err is None else err.data_ptr()
        base = self._own
        keys, ids = self.cand[0], self.cand[1]
        _lib.call("aether_csa_local_candidates", index_q.data_ptr(), index_weight.data_ptr(),
                  cache.idx_pages.data_ptr(), page_table.data_ptr(), page_table.shape[1], cache.num_pages,
                  nblocks.data_ptr(), self.max_nb, rademacher_diag(INDEX_DIM, cache.seed, dev).data_ptr(), B,
                  cache.bits, int(self.top_k), int(id_base), keys.data_ptr(), ids.data_ptr(), self.ws.data_ptr(),
                  ep, st)
        # keys then ids: 2B rows of n words into column rank * n of [2B][G n]
        _lib.call("aether_peer_push", self.cand.data_ptr(), 2 * B, n * 4, n * 4,
                  ctypes.cast(self._bases, ctypes.c_void_p), G, self.rank, self.off_k, G * n * 4,
                  self.rank * n * 4, 0, 1, st)
        _lib.call("aether_peer_wait", base, G, 0, ep, st)
        po = self.part.data_ptr()
        _lib.call("aether_csa_attend_candidates", q.data_ptr(), sink.data_ptr(), window.data_ptr(),
                  window_len.data_ptr(), cache.kv_pages.data_ptr(), page_table.data_ptr(), page_table.shape[1],
                  cache.num_pages, nblocks.data_ptr(), page_table.shape[1] * PAGE,
                  rademacher_diag(HEAD_DIM, cache.seed, dev).data_ptr(), base + self.off_k, base + self.off_i,
                  G * n, G * n, int(id_base), B, H, window.shape[1], cache.bits, int(self.top_k),
                  float(softmax_scale), None, self.sel.data_ptr(), po, po + self.o_bytes, ep, st)
        _lib.call("aether_peer_push", po, 1, self.slot, self.slot, ctypes.cast(self._bases, ctypes.c_void_p), G,
                  self.rank, self.off_p, self.slot, self.rank * self.slot, 1, 0, st)
        _lib.call("aether_peer_wait", base, G, 1, ep, st)
        _lib.call("aether_lse_merge_strided", base + self.off_p, base + self.off_p + self.o_bytes, self.slot // 4,
                  self.slot // 4, sink.data_ptr(), G, B, H, self.out.data_ptr(), st)
        return self.out, self.sel

    def close(self) -> None:
        """Release the buffers (collective: every rank calls it)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)  # no rank still reads or writes a buffer
        for pp in self._opened:
            _lib.call("aether_cp_buffer_close", pp)
        self._opened = []
        _lib.call("aether_cp_buffer_destroy", self._own)
        self._own = None
