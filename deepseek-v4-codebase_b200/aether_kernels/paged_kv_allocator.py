"""Two-tier (HBM / host RAM) LRU page allocator with disk spill.

API-compatible with the reference's ``aether_kernels.paged_kv_allocator``
(aether_kernels/paged_kv_allocator.py:37-252): ``PageHandle``,
``PagedKVAllocator(num_device_pages, num_host_pages, page_shape, dtype,
device, write_to_disk, read_from_disk)`` with ``allocate`` / ``append_page`` /
``load_pages`` / ``free`` / ``device_pages_used`` / ``host_pages_used``, the
same LRU policy (device -> host on device pressure, host -> ``write_to_disk``
on host pressure, page-in on ``load_pages``), the same handle bookkeeping
(``page_slots[i]`` is ``(device_slot, None)``, ``(None, host_slot)`` or
``(None, None)`` when on disk) and the same error types and messages.

What differs is the storage.  The reference keeps a Python list of
per-page tensor dicts; here each named stream is ONE contiguous pool
``[num_pages, *page_shape[name]]`` (pinned on the host side when the device
is CUDA), so ``pool(name)`` is directly a page pool that the paged decode
kernels index with a page table, and a page moves between tiers with one
copy per stream.  With ``page_shape = quantized_page_shape(bits)`` the pools
are the 64-entry TurboQuant pages (``[64 code rows][64 fp32 scales]``) that
``csa_decode_paged`` / ``hca_decode_paged`` read, so evicted pages stay
quantized (a quarter or an eighth of the reference's de-quantized bytes).

``page_table(handles)`` pages every page of a batch in, keeps them resident
for the call, and returns the int32 ``[B, max_pages]`` table the kernels take.
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

PAGE = 64


@dataclass
class PageHandle:
    """Per-sequence handle (aether_kernels/paged_kv_allocator.py:37-43):
    ``page_slots[i]`` = (device_slot, host_slot) of logical page i; at most
    one is set, both None while the page lives on disk."""

    seq_id: str
    page_slots: List[Tuple[Optional[int], Optional[int]]] = field(default_factory=list)


def quantized_page_shape(bits: int, with_index: bool = True, head_dim: int = 128,
                         index_dim: int = 64) -> Dict[str, Tuple[int, ...]]:
    """Page shape (dtype uint8) of the TurboQuant paged cache: ``kv`` holds
    64 main entries, ``idx`` 64 indexer keys, each as 64 code rows of
    dim*bits/8 bytes followed by 64 fp32 scales."""
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    shape = {"kv": (PAGE * head_dim * bits // 8 + PAGE * 4,)}
    if with_index:
        shape["idx"] = (PAGE * index_dim * bits // 8 + PAGE * 4,)
    return shape


class PagedKVAllocator:
    """Two-tier LRU page pool: device HBM and host RAM, spilling to disk.

    Thread-safe via one lock (as aether_kernels/paged_kv_allocator.py:82).
    """

    def __init__(
        self,
        num_device_pages: int,
        num_host_pages: int,
        page_shape: Dict[str, Tuple[int, ...]],
        dtype: torch.dtype = torch.float16,
        device="cuda",
        write_to_disk: Optional[Callable[[str, Dict[str, torch.Tensor]], None]] = None,
        read_from_disk: Optional[Callable[[str], Dict[str, torch.Tensor]]] = None,
    ) -> None:
        self._lock = threading.Lock()
        self._dtype = dtype
        self._device = torch.device(device)
        self._page_shape = {k: tuple(v) for k, v in page_shape.items()}
        self._write_to_disk = write_to_disk
        self._read_from_disk = read_from_disk
        pin = self._device.type == "cuda"
        self._dev: Dict[str, torch.Tensor] = {
            n: torch.zeros((num_device_pages, *s), dtype=dtype, device=self._device)
            for n, s in self._page_shape.items()}
        self._host: Dict[str, torch.Tensor] = {
            n: torch.zeros((num_host_pages, *s), dtype=dtype, pin_memory=pin)
            for n, s in self._page_shape.items()}
        # free lists pop from the end: slot 0 is handed out first
        self._device_free: List[int] = list(range(num_device_pages - 1, -1, -1))
        self._host_free: List[int] = list(range(num_host_pages - 1, -1, -1))
        self._device_lru: "OrderedDict[int, str]" = OrderedDict()   # slot -> page key, oldest first
        self._host_lru: "OrderedDict[int, str]" = OrderedDict()
        self._page_map: Dict[str, Tuple[Optional[int], Optional[int]]] = {}
        self._page_owner: Dict[str, Tuple[PageHandle, int]] = {}

    # ------------------------------------------------------------ properties
    @property
    def num_device_pages(self) -> int:
        return next(iter(self._dev.values())).shape[0] if self._dev else 0

    @property
    def num_host_pages(self) -> int:
        return next(iter(self._host.values())).shape[0] if self._host else 0

    @property
    def page_shape(self) -> Dict[str, Tuple[int, ...]]:
        return dict(self._page_shape)

    def pool(self, name: str) -> torch.Tensor:
        """The device pool of stream ``name``: [num_device_pages, *page_shape]."""
        return self._dev[name]

    def as_cache(self, bits: int, seed: int = 42):
        """The device pools of a ``quantized_page_shape(bits)`` allocator as a
        ``TurboQuantPagedCache`` the paged decode entry points accept."""
        from .paged import TurboQuantPagedCache
        return TurboQuantPagedCache.from_pools(self._dev["kv"], self._dev.get("idx"), bits, seed)

    # ------------------------------------------------------------ public API
    def allocate(self, seq_id: str) -> PageHandle:
        """Reserve a sequence handle; no pages are allocated yet."""
        return PageHandle(seq_id=seq_id)

    def append_page(self, handle: PageHandle, page_tensors: Dict[str, torch.Tensor]) -> None:
        """Append one page to ``handle``'s sequence (paged_kv_allocator.py:116-132)."""
        page_index = len(handle.page_slots)
        key = self._key(handle.seq_id, page_index)
        with self._lock:
            slot = self._alloc_device_page(key)
            for name, t in page_tensors.items():
                self._dev[name][slot].copy_(t)
            self._device_lru[slot] = key
            self._page_map[key] = (slot, None)
            handle.page_slots.append((slot, None))
            self._page_owner[key] = (handle, page_index)

    def append_slot(self, handle: PageHandle) -> int:
        """Append one page without copying data and return its device slot,
        for writers that fill the pool in place (``tq_encode_into_pages``)."""
        page_index = len(handle.page_slots)
        key = self._key(handle.seq_id, page_index)
        with self._lock:
            slot = self._alloc_device_page(key)
            self._device_lru[slot] = key
            self._page_map[key] = (slot, None)
            handle.page_slots.append((slot, None))
            self._page_owner[key] = (handle, page_index)
        return slot

    def load_pages(self, handle: PageHandle,
                   page_range: Optional[Tuple[int, int]] = None) -> List[Dict[str, torch.Tensor]]:
        """Device-resident copies of the pages in ``page_range``; pages on the
        host or on disk are paged in first (paged_kv_allocator.py:134-182)."""
        start, stop = page_range if page_range is not None else (0, len(handle.page_slots))
        out = []
        with self._lock:
            # copy each page as it arrives: a range larger than the device
            # pool evicts its own earlier pages
            for i in range(start, stop):
                s = self._page_in(handle, i)
                out.append({n: self._dev[n][s].clone() for n in self._page_shape})
        return out

    def device_slots(self, handle: PageHandle, page_range: Optional[Tuple[int, int]] = None) -> List[int]:
        """Page ``page_range`` in and return the device slots (no copies)."""
        start, stop = page_range if page_range is not None else (0, len(handle.page_slots))
        with self._lock:
            return [self._page_in(handle, i) for i in range(start, stop)]

    def page_table(self, handles: Sequence[PageHandle], max_pages: Optional[int] = None,
                   device=None) -> torch.Tensor:
        """Page in every page of ``handles`` and return the int32 table
        [len(handles), max_pages] of device slots (unused entries 0).  The
        batch's pages must fit in the device pool together: its resident
        pages are touched first so paging in the rest evicts none of them."""
        counts = [len(h.page_slots) for h in handles]
        width = max(counts + [1]) if max_pages is None else int(max_pages)
        if max(counts + [0]) > width:
            raise ValueError(f"a sequence holds {max(counts)} pages, more than max_pages={width}")
        if sum(counts) > self.num_device_pages:
            raise MemoryError(f"batch needs {sum(counts)} device pages, pool holds {self.num_device_pages}")
        rows = []
        with self._lock:
            for h in handles:
                for dev, _ in h.page_slots:
                    if dev is not None:
                        self._device_lru.move_to_end(dev)
            for h in handles:
                rows.append([self._page_in(h, i) for i in range(len(h.page_slots))])
        table = torch.zeros(len(handles), width, dtype=torch.int32)
        for b, r in enumerate(rows):
            if r:
                table[b, : len(r)] = torch.tensor(r, dtype=torch.int32)
        return table.to(device if device is not None else self._device)

    def free(self, handle: PageHandle) -> None:
        """Release every page of ``handle`` (paged_kv_allocator.py:184-200)."""
        with self._lock:
            for page_index, (dev, host) in enumerate(handle.page_slots):
                key = self._key(handle.seq_id, page_index)
                if dev is not None:
                    self._device_free.append(dev)
                    self._device_lru.pop(dev, None)
                if host is not None:
                    self._host_free.append(host)
                    self._host_lru.pop(host, None)
                self._page_map.pop(key, None)
                self._page_owner.pop(key, None)
            handle.page_slots.clear()

    def device_pages_used(self) -> int:
        with self._lock:
            return len(self._device_lru)

    def host_pages_used(self) -> int:
        with self._lock:
            return len(self._host_lru)

    # ------------------------------------------------------------- internals
    @staticmethod
    def _key(seq_id: str, page_index: int) -> str:
        return f"{seq_id}:{page_index}"

    def _set_owner_slots(self, key: str, slots: Tuple[Optional[int], Optional[int]]) -> None:
        self._page_map[key] = slots
        owner = self._page_owner.get(key)
        if owner is not None:
            handle, page_index = owner
            handle.page_slots[page_index] = slots

    def _page_in(self, handle: PageHandle, page_index: int) -> int:
        """Device slot of one page, paging it in from host or disk (lock held)."""
        key = self._key(handle.seq_id, page_index)
        dev, host = self._page_map.get(key, (None, None))
        if dev is not None:
            self._device_lru.move_to_end(dev)
            return dev
        if host is not None:
            dev = self._alloc_device_page(key)
            for n in self._page_shape:
                self._dev[n][dev].copy_(self._host[n][host], non_blocking=True)
            self._host_free.append(host)
            self._host_lru.pop(host, None)
        else:
            if self._read_from_disk is None:
                raise RuntimeError(
                    f"Page {key} has been evicted to disk but no read_from_disk handler was provided.")
            data = self._read_from_disk(key)
            dev = self._alloc_device_page(key)
            for n in self._page_shape:
                self._dev[n][dev].copy_(data[n])
        self._device_lru[dev] = key
        self._set_owner_slots(key, (dev, None))
        return dev

    def _alloc_device_page(self, key: str) -> int:
        """A free device slot, evicting the LRU device page to host if needed."""
        if self._device_free:
            return self._device_free.pop()
        if not self._device_lru:
            raise MemoryError("Device KV page pool has no pages to evict.")
        slot, victim = self._device_lru.popitem(last=False)
        host = self._alloc_host_page(victim)
        for n in self._page_shape:
            self._host[n][host].copy_(self._dev[n][slot])
        self._host_lru[host] = victim
        self._set_owner_slots(victim, (None, host))
        return slot

    def _alloc_host_page(self, key: str) -> int:
        """A free host slot, spilling the LRU host page to disk if needed."""
        if self._host_free:
            return self._host_free.pop()
        if not self._host_lru:
            raise MemoryError("Both device and host KV page pools are full and no host page can be evicted.")
        if self._write_to_disk is None:
            raise MemoryError(
                "Host KV page pool is full but no write_to_disk handler was provided; "
                "increase num_host_pages or supply write_to_disk.")
        slot, victim = self._host_lru.popitem(last=False)
        self._write_to_disk(victim, {n: self._host[n][slot].clone() for n in self._page_shape})
        self._set_owner_slots(victim, (None, None))
        return slot
