"""Disk-backed prefix store for the quantized paged KV cache.

The reference keeps reusable prompt prefixes on disk with
``OnDiskPrefixKVStore`` (aether_pipeline/serving.py:174-338): the compressed
CSA/HCA entries up to the last complete compression block, optionally the
sliding-window (SWA) state, an ``index.json`` keyed by a SHA-256 of the
reusable tokens, and a restore plan that tells the serving layer what it must
recompute.  It stores de-quantized torch tensors (``torch.save`` of the
engine's compressed dict, aether_2b/serving.py:940-964).

``QuantizedPrefixStore`` keeps that interface -- ``save_prefix``,
``lookup_prefix``, ``load_swa_state``, ``make_restore_plan``, the same
metadata fields, layout checks, hash and plan rules -- but what it persists
is the quantized pages themselves: each layer's index and main pages
(TurboQuant codes + fp32 scales, the ``TurboQuantPagedCache`` page layout)
are written as raw page bytes in logical order, one file per prefix, and
``load_pages`` copies them back into free pages of any cache with the same
page format, returning the page-table rows.  Nothing is decoded or
re-encoded on either side, so a restored prefix is bit-identical, and it
takes about a quarter (4-bit) or a half (8-bit) of the bytes of the
reference's bf16 entries.

File format ``<hash>.pages.bin``: for every layer (in the order of the
metadata's ``layers`` list) and every stream (``idx`` then ``kv``, where
present), ``num_pages`` pages of ``page_bytes`` each, back to back.  The
layout of that file is recorded in the index entry.
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import asdict, dataclass, field
from enum import Enum
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch

PAGE = 64


class SWACacheMode(str, Enum):
    """How much sliding-window state a saved prefix keeps (serving.py:17-20)."""

    FULL = "full"
    PERIODIC = "periodic"
    ZERO = "zero"


@dataclass(frozen=True)
class HybridCacheLayout:
    """Compression ratios, window and depth a prefix was built with
    (serving.py:23-43).  A prefix is reusable up to a multiple of the least
    common multiple of the two compression ratios."""

    csa_compression: int
    hca_compression: int
    window_size: int
    num_layers: int

    @property
    def block_tokens(self) -> int:
        return math.lcm(self.csa_compression, self.hca_compression)

    @property
    def csa_tokens_per_block(self) -> int:
        return self.block_tokens // self.csa_compression

    @property
    def hca_tokens_per_block(self) -> int:
        return self.block_tokens // self.hca_compression

    def full_block_prefix(self, token_count: int) -> int:
        return (token_count // self.block_tokens) * self.block_tokens


@dataclass
class PrefixCacheMetadata:
    """Index record of one saved prefix (serving.py:46-57), plus the page
    layout of its quantized pages."""

    prefix_hash: str
    prefix_token_count: int
    reusable_token_count: int
    swa_mode: str
    window_size: int
    num_layers: int
    csa_compression: int
    hca_compression: int
    checkpoint_stride: int
    files: Dict[str, str] = field(default_factory=dict)
    # page layout of files["pages"]: per layer {"name", "bits", "nblocks",
    # "num_pages", "streams": {stream: page_bytes}}
    layers: List[Dict[str, object]] = field(default_factory=list)


@dataclass
class RestorePlan:
    """What the serving layer reloads and what it recomputes (serving.py:60-68)."""

    reusable_prefix_tokens: int
    recompute_start_token: int
    compressed_prefix_tokens: int
    needs_tail_recompute: bool
    swa_mode: str
    load_swa_checkpoint_from: Optional[int] = None
    restore_last_window_tokens: Optional[int] = None


@dataclass
class LayerPages:
    """One layer's share of a prefix: the cache holding its pages and the
    physical page ids of its logical pages 0 .. ceil(nblocks / 64) - 1."""

    cache: object  # TurboQuantPagedCache (or anything with kv_pages / idx_pages / bits)
    page_ids: Sequence[int]
    nblocks: int


class QuantizedPrefixStore:
    """Prefix store whose compressed payload is the quantized page bytes."""

    def __init__(self, root_dir: str, layout: HybridCacheLayout, swa_mode: SWACacheMode = SWACacheMode.PERIODIC,
                 checkpoint_stride: int = 4096) -> None:
        self.root_dir = Path(root_dir)
        self.layout = layout
        self.swa_mode = SWACacheMode(swa_mode)
        self.checkpoint_stride = int(checkpoint_stride)
        self.root_dir.mkdir(parents=True, exist_ok=True)
        self.index_path = self.root_dir / "index.json"
        if not self.index_path.exists():
            self._store_index({})

    # ------------------------------------------------------------ index
    def _load_index(self) -> Dict[str, Dict[str, object]]:
        return json.loads(self.index_path.read_text()) if self.index_path.exists() else {}

    def _store_index(self, index: Dict[str, Dict[str, object]]) -> None:
        tmp = self.index_path.with_name(self.index_path.name + ".tmp")
        tmp.write_text(json.dumps(index, indent=1, sort_keys=True))
        tmp.replace(self.index_path)  # atomic on POSIX: readers see the old or the new index

    def _check_layout(self, md: PrefixCacheMetadata) -> None:
        for got, want, what in ((md.csa_compression, self.layout.csa_compression, "CSA compression"),
                                (md.hca_compression, self.layout.hca_compression, "HCA compression"),
                                (md.window_size, self.layout.window_size, "SWA window size"),
                                (md.num_layers, self.layout.num_layers, "Layer count")):
            if got != want:
                raise ValueError(f"{what} in cache metadata does not match the active layout")

    @staticmethod
    def prefix_hash(token_ids: Iterable[int]) -> str:
        """SHA-256 over the token ids as little-endian u32 (the key the
        reference's store uses)."""
        h = hashlib.sha256()
        h.update(b"".join(int(t).to_bytes(4, "little", signed=False) for t in token_ids))
        return h.hexdigest()

    def checkpoint_token(self, reusable_tokens: int) -> int:
        """Token at which a PERIODIC store checkpoints the SWA state: the
        last multiple of the stride, or the whole prefix if shorter."""
        s = self.checkpoint_stride
        return reusable_tokens if reusable_tokens <= s else (reusable_tokens // s) * s

    # ------------------------------------------------------------- save
    def save_prefix(self, token_ids: List[int], layers: Dict[str, LayerPages],
                    swa_state: Optional[Dict[str, torch.Tensor]] = None) -> PrefixCacheMetadata:
        """Persist the quantized pages of every layer of a prefix (and the SWA
        state the mode keeps).  ``layers`` maps a layer name to its pages."""
        reusable = self.layout.full_block_prefix(len(token_ids))
        if reusable <= 0:
            raise ValueError(f"Prefix of length {len(token_ids)} does not contain a full compression block of "
                             f"{self.layout.block_tokens} tokens")
        key = self.prefix_hash(token_ids[:reusable])
        md = PrefixCacheMetadata(key, len(token_ids), reusable, self.swa_mode.value, self.layout.window_size,
                                 self.layout.num_layers, self.layout.csa_compression, self.layout.hca_compression,
                                 self.checkpoint_stride)
        pages_path = self.root_dir / f"{key}.pages.bin"
        with open(pages_path.with_name(pages_path.name + ".tmp"), "wb") as f:
            for name, lp in layers.items():
                npg = (int(lp.nblocks) + PAGE - 1) // PAGE
                ids = torch.as_tensor(list(lp.page_ids)[:npg], dtype=torch.long)
                if ids.numel() != npg:
                    raise ValueError(f"layer {name}: {npg} pages needed for {lp.nblocks} blocks, got {ids.numel()}")
                streams = {}
                for sname in ("idx", "kv"):
                    pool = getattr(lp.cache, f"{sname}_pages", None)
                    if pool is None:
                        continue
                    # one gather per stream, then one device->host copy
                    f.write(pool[ids.to(pool.device)].cpu().contiguous().numpy().tobytes())
                    streams[sname] = int(pool.shape[1])
                md.layers.append({"name": name, "bits": int(lp.cache.bits), "nblocks": int(lp.nblocks),
                                  "num_pages": npg, "streams": streams})
        pages_path.with_name(pages_path.name + ".tmp").replace(pages_path)
        md.files["pages"] = pages_path.name
        if swa_state and self.swa_mode != SWACacheMode.ZERO:
            if self.swa_mode == SWACacheMode.FULL:
                p = self.root_dir / f"{key}.swa_full.pt"
                torch.save(swa_state, p)
                md.files["swa_full"] = p.name
            else:
                ck = self.checkpoint_token(reusable)
                p = self.root_dir / f"{key}.swa_ckpt_{ck}.pt"
                torch.save({"token_offset": ck, "state": swa_state}, p)
                md.files["swa_periodic"] = p.name
        index = self._load_index()
        index[key] = asdict(md)
        self._store_index(index)
        return md

    # ------------------------------------------------------------- load
    def lookup_prefix(self, token_ids: List[int]) -> Optional[PrefixCacheMetadata]:
        reusable = self.layout.full_block_prefix(len(token_ids))
        if reusable <= 0:
            return None
        rec = self._load_index().get(self.prefix_hash(token_ids[:reusable]))
        if rec is None:
            return None
        md = PrefixCacheMetadata(**rec)
        self._check_layout(md)
        return md

    def load_pages(self, md: PrefixCacheMetadata, caches: Dict[str, object],
                   page_ids: Optional[Dict[str, Sequence[int]]] = None,
                   generator: Optional[torch.Generator] = None) -> Dict[str, Tuple[torch.Tensor, int]]:
        """Copy a saved prefix's pages into ``caches`` (layer name -> cache
        with the saved page format).  Pages go to ``page_ids[name]`` when
        given, else to pages taken from the cache's free list.  Returns layer
        name -> (int32 page-table row, nblocks)."""
        self._check_layout(md)
        raw = (self.root_dir / md.files["pages"]).read_bytes()
        off, out = 0, {}
        for rec in md.layers:
            name, npg = rec["name"], int(rec["num_pages"])
            cache = caches[name]
            if int(cache.bits) != int(rec["bits"]):
                raise ValueError(f"layer {name}: saved with {rec['bits']}-bit pages, cache holds {cache.bits}-bit")
            ids = (list(page_ids[name]) if page_ids is not None else cache.alloc_pages(npg, generator))[:npg]
            if len(ids) != npg:
                raise ValueError(f"layer {name}: {npg} pages needed, {len(ids)} given")
            idt = torch.as_tensor(ids, dtype=torch.long)
            for sname, pb in rec["streams"].items():
                pool = getattr(cache, f"{sname}_pages", None)
                if pool is None or int(pool.shape[1]) != int(pb):
                    raise ValueError(f"layer {name}: stream {sname} page format differs from the saved one")
                n = npg * int(pb)
                host = torch.frombuffer(bytearray(raw[off: off + n]), dtype=torch.uint8).view(npg, int(pb))
                if pool.is_cuda:
                    host = host.pin_memory()
                pool[idt.to(pool.device)] = host.to(pool.device, non_blocking=True)
                off += n
            out[name] = (torch.tensor(ids, dtype=torch.int32), int(rec["nblocks"]))
        if off != len(raw):
            raise ValueError(f"{md.files['pages']}: {len(raw)} bytes on disk, layout describes {off}")
        return out

    def load_swa_state(self, md: PrefixCacheMetadata) -> Optional[Dict[str, torch.Tensor]]:
        self._check_layout(md)
        mode = SWACacheMode(md.swa_mode)
        if mode == SWACacheMode.FULL and "swa_full" in md.files:
            return torch.load(self.root_dir / md.files["swa_full"], map_location="cpu", weights_only=False)
        if mode == SWACacheMode.PERIODIC and "swa_periodic" in md.files:
            return torch.load(self.root_dir / md.files["swa_periodic"], map_location="cpu",
                              weights_only=False)["state"]
        return None

    def make_restore_plan(self, prefix_tokens: int) -> RestorePlan:
        """FULL restores everything up to the reusable prefix; PERIODIC
        restores the compressed entries and the SWA checkpoint and recomputes
        from the checkpoint; ZERO recomputes the last window of every layer
        (serving.py:306-338)."""
        reusable = self.layout.full_block_prefix(prefix_tokens)
        window = self.layout.window_size
        if self.swa_mode == SWACacheMode.FULL:
            start, ckpt = reusable, None
        elif self.swa_mode == SWACacheMode.PERIODIC:
            start = ckpt = self.checkpoint_token(reusable)
        else:
            start, ckpt = max(0, prefix_tokens - window * self.layout.num_layers), None
        return RestorePlan(reusable_prefix_tokens=reusable, recompute_start_token=start,
                           compressed_prefix_tokens=reusable, needs_tail_recompute=start != prefix_tokens,
                           swa_mode=self.swa_mode.value, load_swa_checkpoint_from=ckpt,
                           restore_last_window_tokens=window)
